"""Benchmark of the decode hot path on B200 (one JSON line on rank 0).

Workload (the config the metric is quoted on): the q4nx
W4A16 GEMV sweep over a dense GQA 3B decoder's projection shapes -- QKV
2560->3584, O 2560->2560, gate+up 2560->16384, down 8192->2560 -- for all 40
layers, batch 1.  One step = the 160 GEMVs of one decode step's weight stream
(1.966 GB, larger than L2), issued in decode order from one CUDA graph.
Synthetic seeded weights with the BASELINE distributions (codes uniform 0..15,
d = |N(0,.02)|, m = -|N(0,.02)|), x ~ N(0,1) bf16.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 (torchrun): every rank streams its own full sweep (weak scaling, no
data-path collective); time = max over ranks; value = all ranks' bytes / time.
`--impl reference` times the reference's own CPU GEMV (designs/granite_gemv/
cpu_baseline.cpp, compiled unmodified into oracle/_ref/) on this host's cores.
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
# that stream from DRAM (ncu capture summarised in profiles/q4nx_gemv_b1_one_layer.md)
GEMV_DRAM_RATIO = 1.003
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


def measure_tc_gemm(torch, ops, gen, device, tensor_peak: float, steps: int) -> list:
    """Tensor-core GEMM (b2_q4_gemm / b2_q4_swiglu_gemm): config-5 MLP shapes at batch 256
    (hidden 1024, intermediate 3584) and config-4 projections at batch 32.  A weight
    pool above L2 is rotated; algorithmic bytes = the q4 tiles, flops = 2*B*N*K."""
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

        def calls(ws_=ws_, x=x, y=y, wsb=wsb, n_t=n_t, k_t=k_t, swiglu=swiglu):
            for g_, u_ in ws_:
                if swiglu:
                    ops.q4_swiglu_gemm(g_, u_, n_t, k_t, x, out=y, workspace=wsb)
                else:
                    ops.q4_gemm(g_, n_t, k_t, x, out=y, workspace=wsb)

        g = graph_of(torch, calls)
        t_ms = time_graph(torch, g, max(5, steps // 50), 3) / pool
        flops = 2 * bsz * n_t * 32 * k_t * 256 * (2 if swiglu else 1)
        out.append({"case": name, "batch": bsz, "us": round(t_ms * 1e3, 2), "gbs": round(per / (t_ms * 1e-3) / 1e9, 1),
                    "tflops": round(flops / (t_ms * 1e-3) / 1e12, 1),
                    "frac_of_measured_tensor": round(flops / (t_ms * 1e-3) / 1e12 / tensor_peak, 3)})
        del g, ws_
        torch.cuda.empty_cache()
    return out


def measure_decode(torch, world: int, rank: int, batch: int, ctx: int, steps: int, warmup: int,
                   program: bool = False) -> dict:
    """Config 4: the full 40-layer decode step at `batch` tokens, context `ctx`, TP over `world` ranks.

    program=True (single GPU, batch <= 8): the persistent decode program + lm_head launch."""
    import torch.distributed as dist
    from llmnputest_b200.decode import GRANITE_3B, Q4Decoder
    from llmnputest_b200.tp import ShardPlan, TPDecoder, shard_weights

    cfg = GRANITE_3B
    if world == 1:
        dec = Q4Decoder(cfg, batch, ctx, seed=11)
    else:
        full_dec = Q4Decoder(cfg, 1, 1, seed=11)  # weights only; the KV cache lives in the TP decoder
        plan = ShardPlan(cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.hidden, cfg.intermediate, cfg.vocab,
                         world, rank)
        dec = TPDecoder(cfg, batch, ctx, shard_weights(full_dec.w, plan), plan)
        del full_dec
        torch.cuda.empty_cache()
    dec.pos.fill_(ctx - 1)  # attend over the full context
    dec.x_in.normal_()
    try:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            dec.step()
        torch.cuda.current_stream().wait_stream(s)
        g = dec.capture(program=True) if program else None
        if g is None:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                dec.step()
        run, how = g.replay, ("persistent program, cuda graph" if program else
                              ("tcgen05 GEMM, cuda graph" if getattr(dec, "use_gemm", False) else "cuda graph"))
    except Exception as e:  # capture of the collectives failed: time the eager step instead
        torch.cuda.synchronize()
        run, how = dec.step, f"eager ({type(e).__name__})"
    for _ in range(warmup):
        run()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        run()
    b.record()
    b.synchronize()
    ms = a.elapsed_time(b) / steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    wb = cfg.weight_bytes()
    kv = batch * ctx * cfg.n_kv_heads * cfg.head_dim * 4 * cfg.n_layers
    step_bytes = wb["layers"] + wb["lm_head"] + kv  # algorithmic: every weight and KV byte once
    out = {"batch": batch, "ctx": ctx, "tp": world, "ms_per_step": round(ms, 4), "program": program,
           "tok_s": round(batch / (ms * 1e-3), 1), "how": how,
           "hbm_gbs_per_gpu": round(step_bytes / world / (ms * 1e-3) / 1e9, 1)}
    del dec
    torch.cuda.empty_cache()
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
    try:
        import torch
        from transformers.cache_utils import DynamicCache
        from transformers.models.qwen3_5 import configuration_qwen3_5 as conf
        from transformers.models.qwen3_5 import modeling_qwen3_5 as mq
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
        return {"us_per_layer": round(dt * 1e6, 1), "threads": torch.get_num_threads(),
                "sample": f"transformers {kind} module, float32, batch {bsz}"
                          + ("" if linear else f", ctx {ctx}") + f", {steps} decode steps"}
    except Exception as e:
        return {"error": f"{type(e).__name__}: {str(e)[:200]}"}


def run_b200(args, rank: int, world: int) -> dict | None:
    import torch
    import torch.distributed as dist
    from llmnputest_b200 import ops

    device = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=device)
    gen.manual_seed(1000 + rank)
    pk = peaks()

    calls, step_bytes = build_sweep(torch, ops, args.batch, args.layers, gen, device)

    def sweep():
        for _, w, n_t, k_t, x, y in calls:
            ops.q4_gemv(w, n_t, k_t, x, out=y, prefetch=True)

    g = graph_of(torch, sweep)
    n_launch = len(calls)

    # ---- timed region (value): K replays, barrier + sync both sides, max over ranks
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    with ClockSampler(gpu_uuid(torch)) as clk:
        time.sleep(0.15)  # let the sampler start
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            g.replay()
        b.record()
        b.synchronize()
    ms = a.elapsed_time(b) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    gbs_total = world * step_bytes / (ms * 1e-3) / 1e9
    gbs_per_gpu = step_bytes / (ms * 1e-3) / 1e9

    extras = {}
    if rank == 0 and not args.quick:
        # per-shape GB/s (40 launches of one shape per replay, > L2 except O/QKV pools)
        per_shape = {}
        for name, n_t, k_t in SHAPES:
            sub = [c for c in calls if c[0] == name]
            gs = graph_of(torch, lambda sub=sub: [ops.q4_gemv(w, n, k, x, out=y, prefetch=True) for _, w, n, k, x, y in sub])
            t_ms = time_graph(torch, gs, max(20, args.steps // 10), 3)
            per_shape[name] = round(sum(c[1].numel() for c in sub) / (t_ms * 1e-3) / 1e9, 1)
            del gs
        extras["per_shape_gbs_b1"] = per_shape
        # batch 8 (config 2's other batch size): same weights, 8-token activations
        calls8 = [(n, w, nt, kt, torch.randn(8, kt * 256, device=device, generator=gen).to(torch.bfloat16),
                   torch.empty(8, nt * 32, device=device)) for n, w, nt, kt, _, _ in calls]
        g8 = graph_of(torch, lambda: [ops.q4_gemv(w, n, k, x, out=y, prefetch=True) for _, w, n, k, x, y in calls8])
        t8 = time_graph(torch, g8, max(20, args.steps // 10), 3)
        extras["batch8_gbs"] = round(step_bytes / (t8 * 1e-3) / 1e9, 1)
        del g8, calls8
        # q8 lm_head (config 1): 248320 x 1024, batch 1, 270 MB > L2
        w8 = make_q8_tiles(torch, 7760 * 4, gen, device)
        x8 = torch.randn(1, 1024, device=device, generator=gen).to(torch.bfloat16)
        y8 = torch.empty(1, 248320, device=device)
        gl = graph_of(torch, lambda: ops.q8_gemv(w8, 7760, 4, x8, out=y8))
        tl = time_graph(torch, gl, max(50, args.steps // 5), 5)
        extras["q8_lm_head"] = {"us": round(tl * 1e3, 2), "gbs": round(w8.numel() / (tl * 1e-3) / 1e9, 1),
                                "frac_of_measured_hbm": round(w8.numel() / (tl * 1e-3) / 1e9 / pk["hbm_gbs"], 3)}
        del gl, w8
        extras["attention"] = measure_attention(torch, ops, gen, device, pk["hbm_gbs"], args.steps)
        extras["tc_gemm"] = measure_tc_gemm(torch, ops, gen, device, pk["bf16_tflops"], args.steps)
        if world == 1:  # config 5's single-GPU layer kernels; the other ranks would wait meanwhile
            extras["deltanet"] = measure_deltanet(torch, ops, gen, device, pk["hbm_gbs"], args.steps)
            extras["deltanet_layers"] = measure_deltanet_layers(torch, device, pk["hbm_gbs"], args.steps)
            extras["gated_attention"] = measure_gated_attention(torch, ops, gen, device, pk["hbm_gbs"],
                                                                args.steps)

    # ---- config 4: the full decode step (tensor-parallel across the ranks when N > 1)
    if not args.quick:
        del g
        extras["decode"] = [measure_decode(torch, world, rank, b, 4096, max(10, args.steps // 30), 3)
                            for b in (1, 8, 32)]
        if world == 1:
            extras["decode"] += [measure_decode(torch, world, rank, b, 4096, max(10, args.steps // 30), 3,
                                                program=True) for b in (1, 8)]

    # ---- e2e: host buffers, copies inside the timed region
    xs_host = torch.cat([c[4].reshape(-1) for c in calls]).cpu().pin_memory()
    ys_host = torch.empty(sum(c[5].numel() for c in calls), dtype=torch.float32).pin_memory()
    x_dev = torch.empty_like(xs_host, device=device)
    y_dev = torch.empty(ys_host.numel(), dtype=torch.float32, device=device)
    views, off_x, off_y = [], 0, 0
    for name, w, n_t, k_t, x, y in calls:
        views.append((w, n_t, k_t, x_dev[off_x:off_x + x.numel()].view(x.shape),
                      y_dev[off_y:off_y + y.numel()].view(y.shape)))
        off_x += x.numel()
        off_y += y.numel()

    def sweep_e2e():
        for w, n_t, k_t, x, y in views:
            ops.q4_gemv(w, n_t, k_t, x, out=y, prefetch=True)

    ge = graph_of(torch, sweep_e2e)
    e2e_steps = max(10, args.steps // 10)

    def e2e_step():
        x_dev.copy_(xs_host, non_blocking=True)
        ge.replay()
        ys_host.copy_(y_dev, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for _ in range(args.warmup):
        e2e_step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(e2e_steps):
        e2e_step()
    b.record()
    b.synchronize()
    e2e_ms = a.elapsed_time(b) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_gbs = world * step_bytes / (e2e_ms * 1e-3) / 1e9
    assert ops.device_error() == 0, "a kernel recorded a device-side error"

    if rank != 0:
        return None
    out = {
        "metric": METRIC,
        "value": round(gbs_total, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded q4nx tiles with BASELINE distributions, x ~ N(0,1) bf16)",
        "config": {
            "workload": "config 2: q4nx W4A16 GEMV sweep, QKV 2560->3584 / O 2560->2560 / gate+up 2560->16384 / "
                        "down 8192->2560, 40 layers, batch 1, one CUDA graph per step",
            "batch": args.batch, "layers": args.layers, "bytes_per_step_per_gpu": step_bytes,
            "l2": "inputs larger than L2 (1.97 GB of weights streamed per step)",
            "parallelism": f"replicas x{world} (each rank streams its own weights, no collective)",
        },
        "gpu_launches": n_launch * args.steps,
        "e2e": {"value": round(e2e_gbs, 1), "unit": "GB/s",
                "h2d_bytes_per_step": int(xs_host.numel() * 2), "d2h_bytes_per_step": int(ys_host.numel() * 4)},
        "roofline": {"bound": "hbm", "achieved": round(gbs_per_gpu, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(gbs_per_gpu / pk["hbm_gbs"], 4),
                     "traffic": int(step_bytes / n_launch * GEMV_DRAM_RATIO),
                     "traffic_unit": "DRAM bytes read+written per launch (mean over the sweep's launches): "
                                     "algorithmic bytes x the ncu ratio in profiles/q4nx_gemv_b1_one_layer.md",
                     "kernel": "q4nx_gemv_kernel<q4,NB=1,f32>", "peak_src": pk["src"]},
        "clocks": clk.summary(),
    }
    if world == 1 and not args.quick:  # config 5 as one step, last (see measure_qwen35_step)
        extras["qwen35_step"] = measure_qwen35_step(torch, device, pk["hbm_gbs"], args.steps)
    out.update(extras)
    if world == 1 and not args.no_cpu_baseline:
        cb = run_reference_gemv(iters=20)
        out["cpu_baseline"] = {"value": round(cb["gbs"], 2), "unit": "GB/s", "cores": cb["cores"],
                               "kind": cb["kind"], "sample": cb["sample"]}
    return out


def run_reference(args, rank: int) -> dict | None:
    if rank != 0:
        return None
    t0 = time.time()
    cb = run_reference_gemv(iters=max(1, args.steps // 10), layers=8)
    sec = time.time() - t0
    return {
        "impl": "reference", "metric": METRIC, "value": round(cb["gbs"], 2), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32 (bf16 codes -> fp32 AVX2 FMA)", "data": "synthetic",
        "config": {"workload": "config 2: q4nx W4A16 GEMV sweep shapes, batch 1 (reference CPU GEMV)",
                   "batch": 1},
        "cpu_baseline": {"value": round(cb["gbs"], 2), "unit": "GB/s", "cores": cb["cores"], "kind": cb["kind"],
                         "sample": cb["sample"]},
        "e2e": {"value": round(cb["gbs"], 2), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": round(sec, 1),
    }


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--quick", action="store_true", help="skip the extra per-shape / q8 / batch-8 lines")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        res = run_reference(args, rank)
    else:
        import torch
        torch.cuda.set_device(local)
        if world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        res = run_b200(args, rank, world)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if res is not None:
        print(json.dumps(res), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
