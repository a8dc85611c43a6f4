"""Benchmark of the B200 GWP-0.5 MoT engine: action chunks per second.

One "step" = one GWP-0.5 action chunk of BASELINE config 2 (full MoT, batch 1
per GPU: prompt projection + 30-layer prefix cache + 10 flow-matching Euler
steps), synthetic random-init BF16 weights and seeded synthetic inputs of the
config's shapes. With --gpus N the engine runs as N independent data-parallel
replicas (one process per GPU, no collective); value = all chunks / max-over-
ranks time. The same line carries "config4": BASELINE config 4, 64 requests
per box split 64/N per GPU (strong scaling), timed after the main measurement,
and (one GPU) "config1": one MoT block through wam_b200_block_forward in the
reference's form and BASELINE's literal form, beside the CPU oracle's block,
"vision": the vision front-end (compose / resize / patchify and the Wan VAE
encoder) on config 2's canvas from three camera views, and "text_encoder": the
UMT5-XXL encoder on a 512-token prompt.

  python bench.py [--gpus N --steps K --warmup W]        this engine
  python bench.py --impl reference [...]                 the reference arm: the
      CPU restatement of the reference's path (oracle/) on the host cores

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "wam.cpp_b200"))

METRIC = "action chunks/sec/box at batch 1-64 (1/2/4/8 B200); p50 ms per chunk at batch 1"
UNIT = "action_chunks/s"
SEED = 20261201


def config2(layers: int | None = None):
    from wam_b200 import workload

    g = dataclasses.replace(workload.CONFIG2, flow_shift=1.0)  # sigmas linear 1 -> 0.001 -> 0
    if layers is not None:
        g = dataclasses.replace(g, layers=layers)
    return g


def workload(g, batch: int, weights: str = "bf16") -> dict:
    if weights == "q8_0":
        return dict(workload(g, batch),
                    workload="config5: config 2 with every linear weight Q8_0 (gguf-py rules, "
                             "quantised on the device; GEMMs convert Q8_0 tiles to BF16 in shared "
                             "memory)",
                    weights="synthetic N(0,0.02) BF16 quantised to Q8_0, biases 0",
                    l2="no flush needed: each chunk streams ~10.5 GB of Q8_0 weights (> 126 MB L2)")
    return {"workload": "config2: GWP-0.5-shaped MoT action chunk (prompt projection + prefix "
                        "cache + 10 Euler steps)",
            "layers": g.layers, "hidden": g.hidden, "action_hidden": g.action_hidden,
            "ffn": g.ffn, "heads": g.heads, "visual_tokens": g.visual_tokens,
            "prompt_tokens": g.prompt_tokens, "text_dim": g.text_dim,
            "action_chunk": [g.action_chunk, g.action_dim], "steps": g.steps,
            "batch_per_gpu": batch, "weights": "synthetic N(0,0.02) BF16, biases 0",
            "l2": "no flush needed: each chunk streams 19.7 GB of weights (> 126 MB L2)"}


def peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        import torch

        try:
            self.device = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            self.device = str(device)
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_sample(layers: int, uncached: bool = False, runs: int = 1, warmup: int = 0) -> dict:
    """Times the oracle (the CPU restatement of the reference path) on a bounded
    sample: one config-2 chunk through `layers` of the 30 layers. Cached mode =
    prefix once + 10 action-expert steps (this engine's schedule); un-cached =
    the whole MoT every step, the reference's own CPU behaviour
    (engine.cpp:334-337)."""
    import oracle
    from wam_b200 import workload as wl

    g = config2(layers)
    m = oracle.OracleModel(g, None, seed=SEED, bias_scale=0.0)
    if uncached:
        m.set_uncached(True)
    r = wl.make_request(g, SEED)
    for _ in range(warmup):
        m.predict(r)
    times = []
    for _ in range(runs):
        t0 = time.perf_counter()
        m.predict(r)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"sample_seconds": t, "runs": runs, "layers": layers, "factor": 30 / layers,
            "chunk_seconds_extrapolated": t * 30 / layers, "mode": "uncached" if uncached else "cached",
            "cores": oracle.lib().oracle_threads()}


def cpu_baseline(layers: int) -> dict:
    """The cpu_baseline object of the bench line: cached (value) and the
    labelled un-cached mode, each one bounded sample extrapolated to 30 layers."""
    c = cpu_sample(layers)
    u = cpu_sample(layers, uncached=True)
    return {"value": 1.0 / c["chunk_seconds_extrapolated"], "unit": UNIT, "cores": c["cores"],
            "kind": "port", "sample_seconds": c["sample_seconds"],
            "sample": f"one config-2 chunk (prompt projection, prefix once, 10 Euler steps) through "
                      f"{layers} of 30 layers, F32 OpenMP oracle, {c['sample_seconds']:.2f} s; chunk "
                      f"time extrapolated x{30 / layers:g} ({c['chunk_seconds_extrapolated']:.1f} s/chunk)",
            "uncached": {"value": 1.0 / u["chunk_seconds_extrapolated"], "unit": UNIT,
                         "sample_seconds": u["sample_seconds"],
                         "sample": f"the reference's CPU mode (whole MoT every step): {layers} of 30 "
                                   f"layers, {u['sample_seconds']:.2f} s, extrapolated x{30 / layers:g} "
                                   f"({u['chunk_seconds_extrapolated']:.1f} s/chunk)"}}


def host_cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args) -> None:
    """The reference arm: the CPU restatement of the reference's path on the
    host cores (the reference's own ggml CPU path cannot be built here). Each
    step is one bounded sample (one config-2 chunk through --cpu-layers of the
    30 layers, cached mode); ms_per_step is that sample's measured time, and
    value is the chunk rate extrapolated to 30 layers (field "extrapolation")."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # the CPU arm runs once per box, on rank 0
    layers = args.cpu_layers
    smp = cpu_sample(layers, runs=args.steps, warmup=args.warmup)
    per_chunk = smp["chunk_seconds_extrapolated"]
    value = 1.0 / per_chunk
    unc = cpu_sample(layers, uncached=True)
    cb = {"value": value, "unit": UNIT, "cores": smp["cores"], "kind": "port",
          "cpu_model": host_cpu_model(),
          "sample": f"each step: one config-2 chunk (prompt projection, prefix once, 10 Euler "
                    f"steps) through {layers} of 30 layers with the F32 OpenMP oracle "
                    f"({smp['sample_seconds']:.2f} s median), rate extrapolated x{30 / layers:g}",
          "uncached": {"value": 1.0 / unc["chunk_seconds_extrapolated"], "unit": UNIT,
                       "sample_seconds": unc["sample_seconds"],
                       "sample": "the reference's own CPU mode (whole MoT every step, "
                                 "engine.cpp:334-337), one run of the same sample"}}
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": smp["sample_seconds"] * 1e3,
            "extrapolation": {"measured": f"{layers} of 30 layers per step",
                              "factor": 30 / layers, "ms_per_chunk": per_chunk * 1e3},
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": workload(config2(), 1), "cpu_baseline": cb,
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference's ggml CPU path cannot be built here (llama.cpp b9866 is not "
                    "vendored); this arm times the oracle/ C++ restatement of that path"}
    print(json.dumps(line), flush=True)


def run_op_case(args) -> None:
    """One kernel of the chunk on its own, `--warmup` + `--steps` launches on
    rotating buffers larger than L2: the case the ncu captures in profiles/ use."""
    import torch
    from wam_b200 import ops

    kind, dims = args.op_case.split(":")
    d = [int(v) for v in dims.split(",")]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device="cpu").manual_seed(SEED)
    if kind == "gemm":
        m, n, k = d
        rot = max(2, (256 << 20) // (n * k * 2) + 1)  # > 2x L2 of weights in rotation
        ws = [ops.TiledWeight((torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16).to(dev))
              for _ in range(rot)]
        x = torch.randn(m, k, generator=gen).to(torch.bfloat16).to(dev)
        b = torch.zeros(n, dtype=torch.bfloat16, device=dev)
        y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        sc = ops.Scratch() if args.scratch else None
        fn = lambda i: ops.gemm(x, ws[i % rot], ops.EPI_BIAS, bias=b, out=y, scratch=sc,
                                force_splits=args.force_splits)
        algo = n * k * 2 + m * k * 2 + m * n * 2
    elif kind == "matmul":
        # The same GEMM through torch.matmul (cuBLAS), for comparison on the same box.
        m, n, k = d
        rot = max(2, (256 << 20) // (n * k * 2) + 1)
        ws = [(torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16).to(dev) for _ in range(rot)]
        x = torch.randn(m, k, generator=gen).to(torch.bfloat16).to(dev)
        y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        fn = lambda i: torch.matmul(x, ws[i % rot].T, out=y)
        algo = n * k * 2 + m * k * 2 + m * n * 2
    elif kind == "attention":
        lq, lk, heads = d
        q = torch.randn(1, heads, lq, 128, generator=gen).to(torch.bfloat16).to(dev)
        rot = max(2, (256 << 20) // (heads * lk * 128 * 4) + 1)
        kv = [(torch.randn(1, heads, lk, 128, generator=gen).to(torch.bfloat16).to(dev),
               torch.randn(1, heads, lk, 128, generator=gen).to(torch.bfloat16).to(dev))
              for _ in range(rot)]
        o = torch.empty(lq, heads * 128, dtype=torch.bfloat16, device=dev)
        fn = lambda i: ops.attention(q, kv[i % rot][0], kv[i % rot][1], out=o)
        algo = heads * (2 * lq + 2 * lk) * 128 * 2
    elif kind == "layernorm":
        # LayerNorm + AdaLN modulation (F32 scale / shift) of a token-major
        # BF16 activation, e.g. 49152 x 3072 = the batch-64 prefix rows.
        rows, cols = d
        rot = max(2, (256 << 20) // (rows * cols * 2) + 1)
        xs = [torch.randn(rows, cols, generator=gen).to(torch.bfloat16).to(dev) for _ in range(rot)]
        ys = [torch.empty_like(xs[0]) for _ in range(rot)]
        sc = (torch.randn(cols, generator=gen) * 0.02).to(dev)
        sh = (torch.randn(cols, generator=gen) * 0.02).to(dev)
        fn = lambda i: ops.layernorm(xs[i % rot], sc, sh, out=ys[i % rot])
        algo = rows * cols * 2 * 2 + cols * 4 * 2
    elif kind == "q8quant":
        # BF16 [n, k] weight -> GGML Q8_0 blocks (the config-5 load-time quantiser).
        n, k = d
        rot = max(2, (256 << 20) // (n * k * 2) + 1)
        ws = [(torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16).to(dev) for _ in range(rot)]
        bs = [torch.empty(n * k // 32, 34, dtype=torch.uint8, device=dev) for _ in range(rot)]
        fn = lambda i: ops.q8_quantize(ws[i % rot], out=bs[i % rot])
        algo = n * k * 2 + n * k // 32 * 34
    else:
        raise SystemExit(f"unknown op case {kind}")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            fn(i)
    torch.cuda.synchronize()
    # The timed launches replay as one CUDA graph, so host call overhead does
    # not show up between them.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(args.steps):
            fn(i)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        graph.replay()  # the first replay of a graph pays its upload: untimed
        e0.record()
        graph.replay()
        e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    line = {"op_case": args.op_case, "force_splits": args.force_splits,
            "scratch": bool(args.scratch), "launches": args.steps, "avg_us": round(us, 3),
            "algorithmic_bytes": algo, "GB/s": round(algo / us / 1e3, 1)}
    if kind in ("gemm", "matmul"):
        line["TFLOP/s"] = round(2.0 * d[0] * d[1] * d[2] / us / 1e6, 1)
    print(json.dumps(line))


def run_attention_bench(args) -> None:
    """BF16 flash attention of 48 action + 768 video queries
    over cached K/V of 1280 / 4096 / 16384 keys, 24 heads x 128, batch 1 / 8 /
    64, Q, K, V ~ N(0, 1) (seeded; RoPE is applied before the kernel, so the
    kernel's inputs are plain Q / K / V). Each point replays `--steps` launches
    in a CUDA graph after `--warmup` untimed ones; prints one JSON line."""
    import torch
    from wam_b200 import ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pk = peaks()
    lq, heads = 48 + 768, 24
    points = []
    for lk in (1280, 4096, 16384):
        for B in (1, 8, 64):
            gen = torch.Generator(device=dev).manual_seed(SEED + lk + B)
            q = torch.randn(B, heads, lq, 128, generator=gen, device=dev).to(torch.bfloat16)
            k = torch.randn(B, heads, lk, 128, generator=gen, device=dev).to(torch.bfloat16)
            v = torch.randn(B, heads, lk, 128, generator=gen, device=dev).to(torch.bfloat16)
            o = torch.empty(B * lq, heads * 128, dtype=torch.bfloat16, device=dev)
            stream = torch.cuda.Stream()
            with torch.cuda.stream(stream):
                for _ in range(args.warmup):
                    ops.attention(q, k, v, out=o)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for _ in range(args.steps):
                    ops.attention(q, k, v, out=o)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                e0.record()
                graph.replay()
                e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / args.steps
            flops = 4.0 * B * heads * lq * lk * 128
            byts = 2.0 * B * heads * (2 * lq + 2 * lk) * 128
            points.append({"cache": lk, "batch": B, "avg_us": round(us, 2),
                           "TFLOP/s": round(flops / us / 1e6, 1),
                           "frac_of_bf16_peak": round(flops / us / 1e6 / pk["bf16_tflops"], 3),
                           "GB/s": round(byts / us / 1e3, 1)})
            del q, k, v, o, graph
            torch.cuda.empty_cache()
    print(json.dumps({"bench": "config3 attention microbench (launch_attention: tcgen05 kernel for >= 128 queries)",
                      "queries": lq, "heads": heads, "steps": args.steps, "warmup": args.warmup,
                      "peak_tflops": pk["bf16_tflops"], "peak_source": pk["source"],
                      "points": points}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=15,
                    help="timed chunks (15 = the reference wam-bench repetitions, p50 / p95 over them)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=1, help="requests per GPU per step")
    ap.add_argument("--cpu-layers", type=int, default=2, help="layers in the CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--weights", choices=["bf16", "q8_0"], default="bf16",
                    help="q8_0: BASELINE config 5 (every linear weight Q8_0) instead of config 2")
    ap.add_argument("--op-case", default=None,
                    help="gemm:M,N,K, matmul:M,N,K (torch.matmul, for comparison), "
                         "attention:LQ,LK,HEADS, layernorm:ROWS,COLS or "
                         "q8quant:N,K: run one kernel on a small case "
                         "(for ncu captures) and print its event timing instead of the bench line")
    ap.add_argument("--force-splits", type=int, default=0,
                    help="op case gemm: split-K factor (0 = the planner's choice)")
    ap.add_argument("--scratch", action="store_true",
                    help="op case gemm: split-K partials through a global workspace (as the engine)")
    ap.add_argument("--no-text", action="store_true",
                    help="skip the UMT5 text encoder measurement")
    ap.add_argument("--no-vision", action="store_true",
                    help="skip the vision front-end measurement (stage 1 + VAE encoder)")
    ap.add_argument("--no-config1", action="store_true",
                    help="skip the config-1 single-block point (GPU and CPU) of the bench line")
    ap.add_argument("--config4-requests", type=int, default=64,
                    help="BASELINE config 4: requests per box, split over the GPUs (0 = skip)")
    ap.add_argument("--config4-steps", type=int, default=3,
                    help="timed chunks of the config-4 block per GPU")
    ap.add_argument("--attention-bench", action="store_true",
                    help="BASELINE config 3: the attention microbench over cache length and batch")
    args = ap.parse_args()
    if args.op_case:
        run_op_case(args)
        return
    if args.attention_bench:
        run_attention_bench(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    if args.warmup < 3:
        args.warmup = 3

    import numpy as np
    import torch
    from wam_b200 import dp as dp_host
    from wam_b200 import workload as wl
    from wam_b200.engine import Engine, Req

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    def barrier():
        if dist:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        return dp_host.max_over_ranks(x, dist, device=torch.device("cuda", local))

    g = config2()
    B = args.batch
    eng = Engine(g, seed=SEED, bias_scale=0.0, device=local, max_batch=B, graphs=True,
                 weights=args.weights,
                 prompt_cache=False)
    reqs = []
    for i in range(B):
        r = wl.make_request(g, dp_host.request_seed(SEED, rank, i))
        reqs.append(Req(r.state, r.latent, r.prompt, r.noise))
    stream = torch.cuda.ExternalStream(eng.stream())
    kernels_per_chunk = eng.kernel_launches(B, with_prompt=True)

    # ---- device-resident throughput: inputs staged in HBM before timing
    eng.stage(reqs)
    for _ in range(args.warmup):
        eng.run(B)
    torch.cuda.synchronize()
    barrier()
    events = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("timed")  # lets ncu --nvtx-include "timed/" pick these launches
        with torch.cuda.stream(stream):
            events[0].record()
            for i in range(args.steps):
                eng.run(B)
                events[i + 1].record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    barrier()
    per = [events[i].elapsed_time(events[i + 1]) for i in range(args.steps)]
    total_s = max_over_ranks(sum(per) / 1e3)
    value = dp_host.job_throughput([B * args.steps] * world, total_s)
    out = eng.fetch(reqs)
    assert np.isfinite(out).all(), "non-finite action chunk"

    # ---- end to end through the public C ABI: host inputs -> predict_batch -> host actions
    for _ in range(2):
        eng.predict_batch(reqs)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        eng.predict_batch(reqs)
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e_value = dp_host.job_throughput([B * args.steps] * world, e2e_s)
    A, T, Nt, D = g.action_dim, g.action_chunk, g.prompt_tokens, g.text_dim
    h2d = B * 4 * (A + g.vae_z * 4 * g.visual_tokens + Nt * D + T * A)
    d2h = B * 4 * (T * A + 1)

    eng.stage(reqs)
    eng.run(B)
    phases = eng.phase_ms()
    pk = peaks()
    # Roofline of the dominant kernels: their launches replayed alone inside a
    # CUDA graph (same plans and buffers as the timed chunk); the eager per-op
    # profile after it only gives the breakdown by kind.
    hbm_roof = graph_roofline(eng, B, "denoise", pk, "hbm")
    tc_roof = graph_roofline(eng, B, "prefix", pk, "tensor")
    breakdown_graph = graph_breakdown(eng, B)
    eng.stage(reqs)
    prof = eng.profile(B)
    breakdown = breakdown_from_profile(prof)
    del eng
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    barrier()

    # ---- 64 requests per box, 64 / N per GPU (strong scaling)
    c4 = None
    if args.config4_requests > 0:
        c4 = run_config4(args, g, world, rank, local, barrier, max_over_ranks)
    barrier()
    if dist:
        dist.destroy_process_group()
    if rank != 0:
        return
    cb = None
    c1 = None
    if world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(args.cpu_layers)
        cb["cpu_model"] = host_cpu_model()
    if world == 1 and not args.no_config1:
        c1 = run_config1(local, cpu=not args.no_cpu_baseline)
    vis = None
    if world == 1 and not args.no_vision:
        vis = run_vision(local, cpu=not args.no_cpu_baseline)
    txt = None
    if world == 1 and not args.no_text:
        txt = run_text(local, cpu=not args.no_cpu_baseline)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_s * 1e3 / args.steps,
        "p50_ms_per_chunk": statistics.median(per), "p95_ms_per_chunk": float(np.percentile(per, 95)),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": {**workload(g, B, args.weights), "parallelism": f"dp{world} (replicas, no collective)"},
        "roofline": hbm_roof, "roofline_tensor": tc_roof, "clocks": clocks.summary(),
        "phase_ms": phases, "kernel_breakdown_graph": breakdown_graph,
        "kernel_breakdown_eager": breakdown,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_s * 1e3 / args.steps},
        "gpu_launches": kernels_per_chunk * args.steps,
        "kernels_per_chunk": kernels_per_chunk,
        "config4": c4,
        "config1": c1,
        "vision": vis,
        "text_encoder": txt,
        "cpu_baseline": cb,
    }
    print(json.dumps(line), flush=True)


def block_flops(g, ffn: str) -> float:
    """Algorithmic FLOPs of one config-1 block (2 per MAC): both experts'
    projections (QKV, O, cross Q / K / V / O, FFN up and down; the SiLU-gated
    FFN has twice the up rows) and the joint / cross attention products."""
    H, E, V, T, Nt = g.hidden, g.action_hidden, g.visual_tokens, g.action_chunk, g.prompt_tokens
    fin = 2 if ffn == "swiglu" else 1
    rows = {"v": (V, H, g.ffn), "a": (1 + T, E, g.action_ffn)}
    f = 0.0
    for m, w, ff in rows.values():
        f += 2.0 * m * (3 * H * w + H * w + H * w + H * w + fin * ff * w + w * ff)
        f += 2.0 * Nt * 2 * H * w  # text K / V projection of this expert
    P = 1 + V
    f += 4.0 * P * P * H + 4.0 * T * (P + T) * H  # joint attention (prefix rows, action rows)
    f += 4.0 * (V + 1 + T) * Nt * H  # cross attention of both experts
    return f


def run_config1(dev_index: int = 0, reps: int = 10, cpu: bool = True) -> dict:
    """one MoT block at config-2 widths (768 visual + 1 state
    + 48 action tokens, 512 text tokens as cross-attention keys) through
    wam_b200_block_forward, for the reference's form (LayerNorm AdaLN, GELU
    FFN) and BASELINE's literal form (RMSNorm AdaLN, SiLU-gated FFN). GPU: device
    ms per block (CUDA events around the block's three graphs) and end-to-end ms
    (host inputs and outputs); CPU: the oracle's block_forward on the host cores."""
    import torch
    from wam_b200 import workload as wl
    from wam_b200.engine import Engine

    g = wl.CONFIG1
    x = wl.make_block_inputs(g, SEED)
    out = {"workload": "config1: one MoT block over given hidden states (768 visual, 1 state, "
                       "48 action tokens; 512 text tokens as cross-attention keys)", "variants": {}}
    pk = peaks()
    for ffn, norm in (("gelu", "layernorm"), ("swiglu", "rmsnorm")):
        eng = Engine(g, seed=SEED, bias_scale=0.0, device=dev_index, prompt_cache=False, ffn=ffn,
                     norm=norm, block=True)
        for _ in range(3):
            eng.block_forward(x["t"], x["xv"], x["xa"], x["tv"], x["ta"])
        dev_ms, wall = [], []
        for _ in range(reps):
            t0 = time.perf_counter()
            _, _, ms = eng.block_forward(x["t"], x["xv"], x["xa"], x["tv"], x["ta"], with_time=True)
            wall.append((time.perf_counter() - t0) * 1e3)
            dev_ms.append(ms)
        del eng
        torch.cuda.empty_cache()
        fl = block_flops(g, ffn)
        d = statistics.median(dev_ms)
        rec = {"device_ms_p50": d, "e2e_ms_p50": statistics.median(wall), "gflop": fl / 1e9,
               "tflops": fl / d / 1e9, "frac_of_bf16_peak": fl / d / 1e9 / pk["bf16_tflops"]}
        if cpu:
            import oracle

            om = oracle.OracleModel(g, None, seed=SEED, bias_scale=0.0,
                                    ffn_kind=1 if ffn == "swiglu" else 0)
            om.block(x["t"], x["xv"], x["xa"], x["tv"], x["ta"], norm_kind=1 if norm == "rmsnorm" else 0)
            t0 = time.perf_counter()
            om.block(x["t"], x["xv"], x["xa"], x["tv"], x["ta"], norm_kind=1 if norm == "rmsnorm" else 0)
            rec["cpu_ms"] = (time.perf_counter() - t0) * 1e3
            rec["cpu_cores"] = oracle.lib().oracle_threads()
            rec["cpu_kind"] = "port (F32 OpenMP oracle)"
        out["variants"][f"{ffn}+{norm}"] = rec
    return out


def run_vision(dev_index: int = 0, reps: int = 10, cpu: bool = True) -> dict:
    """The vision front-end at config 2's canvas (768 x 1024, three 640 x 480
    camera views, z = 48): stage 1 (compose / resize / patchify kernel, HBM
    roofline on its input + output bytes) and the Wan VAE encoder (captured
    graph of implicit-GEMM convolutions, tensor roofline on its FLOPs), each
    device-timed with CUDA events on the launching stream after 3 warm-ups;
    e2e = host views in, host latent out (wam_b200_vae_encode). CPU: the
    oracle's stage 1 + encoder on a bounded sample (a 256 x 256 canvas)."""
    import torch
    from wam_b200 import vision
    from wam_b200.workload import VIEWS_CONFIG2, make_views

    W, H, z = 768, 1024, 48
    views = make_views(SEED, VIEWS_CONFIG2)
    dviews = [torch.from_numpy(v).cuda(dev_index) for v in views]
    vae = vision.Vae(W, H, z_dim=z, seed=SEED, device_index=dev_index)
    pix = vision.preprocess(dviews, W, H)
    lat = vae.encode_device(pix)
    for _ in range(3):
        vision.preprocess(dviews, W, H, out=pix)
        vae.encode_device(pix, lat)
    torch.cuda.synchronize()
    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    # Stage 1 takes microseconds: 20 launches captured in one CUDA graph so that
    # the events time the kernels, not the host's launch calls.
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        vision.preprocess(dviews, W, H, out=pix)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for _ in range(20):
                vision.preprocess(dviews, W, H, out=pix)
    torch.cuda.synchronize()
    pre_ms, enc_ms = [], []
    for _ in range(reps):
        e[0].record()
        graph.replay()
        e[1].record()
        vae.encode_device(pix, lat)
        e[2].record()
        torch.cuda.synchronize()
        pre_ms.append(e[0].elapsed_time(e[1]) / 20)
        enc_ms.append(e[1].elapsed_time(e[2]))
    del graph
    wall = []
    for _ in range(reps):
        t0 = time.perf_counter()
        vae.encode(views)
        wall.append((time.perf_counter() - t0) * 1e3)
    pk = peaks()
    pre_bytes = sum(v.nbytes for v in views) + pix.numel() * 4
    p50_pre, p50_enc = statistics.median(pre_ms), statistics.median(enc_ms)
    out = {"workload": "vision front-end: 3 x 640x480 u8 views -> 768x1024 canvas -> "
                       "latent 48x64x48 (synthetic VAE weights)",
           "preprocess": {"device_us_p50": p50_pre * 1e3, "bytes": pre_bytes,
                          "GB/s": pre_bytes / p50_pre / 1e6,
                          "frac_of_hbm": pre_bytes / p50_pre / 1e6 / pk["hbm_gbs"]},
           "vae_encoder": {"device_ms_p50": p50_enc, "gflop": vae.flops / 1e9,
                           "tflops": vae.flops / p50_enc / 1e9,
                           "frac_of_bf16_peak": vae.flops / p50_enc / 1e9 / pk["bf16_tflops"],
                           "launches": vae.launches},
           "e2e_ms_p50": statistics.median(wall),
           "e2e_note": "host views -> host latent: H2D copies, stage 1, encoder graph, D2H"}
    if cpu:
        import oracle
        from oracle import synth

        sw, sh = 256, 256
        weights = synth.make_vae_weights(SEED, z)
        mean, std = vision.vae_synthetic_stats(z)
        t0 = time.perf_counter()
        px = oracle.compose_and_patchify(views, sw, sh)
        oracle.vae_encode(weights, mean, std, z, px, sw, sh)
        dt = time.perf_counter() - t0
        out["cpu"] = {"sample": f"{sw}x{sh} canvas ({sw * sh / (W * H):.4f} of the pixels)",
                      "sample_ms": dt * 1e3,
                      "ms_scaled_to_config2": dt * 1e3 * (W * H) / (sw * sh),
                      "cores": oracle.lib().oracle_threads(), "kind": "port (F32 OpenMP oracle)"}
    vae.close()
    return out


def run_text(dev_index: int = 0, reps: int = 5, cpu: bool = True) -> dict:
    """The UMT5-XXL text encoder (24 layers, 4096 wide, 64 heads, FFN 10240,
    synthetic weights) on a 512-token prompt (config 2's N_t): device ms with
    CUDA events around the captured graph on the launching stream after 2
    warm-ups, tensor roofline on its FLOPs; e2e = host tokens in, host
    embedding out (wam_b200_t5_encode). CPU: the oracle on a bounded sample
    (one layer of the same widths over 64 tokens), scaled by layers x tokens."""
    import numpy as np
    import torch
    from wam_b200.text import T5_XXL, T5Geometry, TextEncoder

    g = T5_XXL
    enc = TextEncoder(g, seed=SEED, device_index=dev_index)
    tok = np.random.default_rng(SEED).integers(0, g.vocab, g.max_tokens).astype(np.int32)
    out = enc.encode_device(tok)
    for _ in range(2):
        enc.encode_device(tok, out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ms = []
    for _ in range(reps):
        e0.record()
        enc.encode_device(tok, out)
        e1.record()
        torch.cuda.synchronize()
        ms.append(e0.elapsed_time(e1))
    wall = []
    for _ in range(reps):
        t0 = time.perf_counter()
        enc.encode(tok)
        wall.append((time.perf_counter() - t0) * 1e3)
    flops, launches = enc.info(g.max_tokens)
    enc.close()
    torch.cuda.empty_cache()
    d = statistics.median(ms)
    pk = peaks()
    rec = {"workload": f"UMT5-XXL encoder, {g.max_tokens} tokens (synthetic weights)",
           "device_ms_p50": d, "gflop": flops / 1e9, "tflops": flops / d / 1e9,
           "frac_of_bf16_peak": flops / d / 1e9 / pk["bf16_tflops"], "launches": launches,
           "e2e_ms_p50": statistics.median(wall),
           "e2e_note": "host token ids -> host [512 x 4096] F32 embedding"}
    if cpu:
        import oracle
        from oracle import synth

        sg = T5Geometry(vocab=1000, hidden=g.hidden, ffn=g.ffn, heads=g.heads, head_dim=64,
                        layers=1, max_tokens=64)
        w = synth.make_t5_weights(SEED, sg)
        t = np.random.default_rng(1).integers(0, sg.vocab, 64).astype(np.int32)
        t0 = time.perf_counter()
        oracle.t5_encode(w, sg, t, sg.max_tokens)
        dt = time.perf_counter() - t0
        rec["cpu"] = {"sample": "1 layer, 64 tokens, XXL widths", "sample_ms": dt * 1e3,
                      "ms_scaled": dt * 1e3 * g.layers * g.max_tokens / 64,
                      "cores": oracle.lib().oracle_threads(), "kind": "port (F32 OpenMP oracle)"}
    return rec


def run_config4(args, g, world, rank, local, barrier, max_over_ranks) -> dict:
    """R independent requests per box (default 64), sharded
    in contiguous blocks of R / N per GPU (wam_b200.dp.shard), one engine per
    GPU running its block as one batch; no collective on the data path. Times
    `--config4-steps` chunks of the whole block after 3 warm-up ones."""
    import torch
    from wam_b200 import dp as dp_host
    from wam_b200 import workload as wl
    from wam_b200.engine import Engine, Req

    R = args.config4_requests
    start, stop = dp_host.shard(R, world, rank)
    b = stop - start
    eng = Engine(g, seed=SEED, bias_scale=0.0, device=local, max_batch=b, graphs=True,
                 weights=args.weights, prompt_cache=False)
    reqs = []
    for i in range(start, stop):
        r = wl.make_request(g, dp_host.request_seed(SEED, 0, i))
        reqs.append(Req(r.state, r.latent, r.prompt, r.noise))
    eng.stage(reqs)
    for _ in range(3):
        eng.run(b)
    stream = torch.cuda.ExternalStream(eng.stream())
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record()
        for _ in range(args.config4_steps):
            eng.run(b)
        e1.record()
    torch.cuda.synchronize()
    t = max_over_ranks(e0.elapsed_time(e1) / 1e3)
    phases = eng.phase_ms()
    # Tensor roofline of this block's prefix GEMMs (visual lane: b x 768 tokens),
    # after the timed chunks, on rank 0's engine only (no collective follows).
    roof = graph_roofline(eng, b, "prefix", peaks(), "tensor", sustained=True) if rank == 0 else None
    del eng
    torch.cuda.empty_cache()
    return {"workload": f"config4: {R} independent config-2 requests per box in contiguous blocks "
                        f"of {R}/{world} per GPU (data parallel, no collective)",
            "requests_per_box": R, "requests_per_gpu": b, "steps": args.config4_steps, "warmup": 3,
            "value": R * args.config4_steps / t, "unit": UNIT, "scaling": "strong",
            "ms_per_step": t * 1e3 / args.config4_steps, "phase_ms_rank0": phases,
            "roofline_tensor_rank0": roof}


def graph_roofline(eng, B, phase, pk, bound, sustained: bool = False) -> dict:
    """Achieved HBM bandwidth (denoise GEMMs, weight streaming) or tensor
    throughput (prefix GEMMs) of one phase's GEMM launches, replayed alone in a
    CUDA graph (wam_b200_profile_graph) and timed with CUDA events on the
    engine's stream."""
    # The tensor-bound GEMMs are the prefix's visual lane (768 tokens per
    # request, the main stream); its state-token lane streams weights.
    r = eng.profile_graph(B, phase, "gemm", reps=5, lane=0 if bound == "tensor" else -1)
    sec = r["ms"] / 1e3
    n = max(r["launches"], 1)
    if bound == "hbm":
        ach = r["bytes"] / sec / 1e9
        out = {"bound": "hbm", "kernel": "gemm_tc_kernel, denoise phase (M = 48 tokens per request)",
               "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": ach / pk["hbm_gbs"],
               "algorithmic_bytes_per_launch": r["bytes"] / n,
               "peak_source": pk["source"] + " HBM copy (burst)"}
        traffic = REPO / "profiles" / "gemm_traffic.json"
        out["traffic"] = (json.loads(traffic.read_text()).get("denoise_bytes_per_launch")
                          if traffic.exists() else None)
        out["traffic_source"] = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of the same GEMM "
                                 "shapes, launch-weighted (profiles/gemm_traffic.json); not measured "
                                 "in this run")
    else:
        ach = r["flops"] / sec / 1e12
        # A phase that runs for seconds (the 64-request block) is held to the
        # sustained (power-capped) cuBLAS rate, a short one to the burst rate.
        peak = pk["bf16_tflops_sustained"] if sustained and pk.get("bf16_tflops_sustained") else pk["bf16_tflops"]
        out = {"bound": "tensor",
               "kernel": "tcgen05 GEMMs of the prefix's visual lane (768 tokens per request): "
                         "CTA-pair, persistent and split-K kernels",
               "achieved": ach, "peak": peak, "unit": "TFLOP/s",
               "frac": ach / peak,
               "peak_source": pk["source"] + " cuBLAS bf16 (" + ("sustained" if peak != pk["bf16_tflops"] else "burst") + ")"}
    out.update({"avg_launch_us": sec / n * 1e6, "launches": r["launches"],
                "timing": f"the chunk's {r['launches']} {phase}-phase GEMM launches"
                          f"{' of the visual lane' if bound == 'tensor' else ''} captured alone in "
                          f"a CUDA graph (same plans, buffers and PDL), CUDA events around 5 replays"})
    return out


def graph_breakdown(eng, B) -> dict:
    """Device time of each (phase, kind) of the chunk with its launches
    replayed alone in a CUDA graph (wam_b200_profile_graph; same plans,
    buffers and PDL as the timed chunk). The kinds' sum falls short of the
    phase times by the boundaries between kinds."""
    from wam_b200.engine import KINDS, PHASES
    out = {}
    for ph in PHASES:
        for kind in KINDS:
            if kind == "sync":
                continue
            try:
                r = eng.profile_graph(B, ph, kind, reps=3)
            except RuntimeError:  # no launch of this kind in this phase
                continue
            if r["launches"] == 0:
                continue
            out[f"{ph}/{kind}"] = {"ms": round(r["ms"], 3), "launches": r["launches"],
                                   "us_per_launch": round(r["ms"] * 1e3 / r["launches"], 2)}
    return dict(sorted(out.items(), key=lambda kv: -kv[1]["ms"]))


def breakdown_from_profile(prof: list[dict]) -> dict:
    """Device time by (phase, kind) and by GEMM shape from the engine's eager
    per-op profile (CUDA events around every op, no graph, no PDL overlap)."""
    total = sum(o["ms"] for o in prof)
    br = {}
    for o in prof:
        k = o["phase"] + "/" + o["kind"]
        br[k] = br.get(k, 0.0) + o["ms"]
    breakdown = {k: {"ms": round(v, 3), "share": round(v / total, 4)} for k, v in
                 sorted(br.items(), key=lambda kv: -kv[1])}
    breakdown["_total_eager_ms"] = round(total, 3)
    shapes = {}
    for o in prof:
        if o["kind"] == "gemm" and o["phase"] in ("denoise", "prefix"):
            m, n, k, sp = o["shape"]
            # sp < 0: the CTA-pair kernel with -sp splits
            key = f'{o["phase"]}:{m}x{n}x{k}/' + (f"p{-sp}" if sp < 0 else f"s{sp}")
            e = shapes.setdefault(key, [0, 0.0, 0.0])
            e[0] += 1
            e[1] += o["ms"]
            e[2] += o["bytes"] if o["phase"] == "denoise" else o["flops"]
    breakdown["_gemm_shapes"] = {
        k: {"launches": v[0], "avg_us": round(v[1] / v[0] * 1e3, 2),
            ("GB/s" if k.startswith("denoise") else "TFLOP/s"):
                round(v[2] / (v[1] / 1e3) / (1e9 if k.startswith("denoise") else 1e12), 1)}
        for k, v in sorted(shapes.items(), key=lambda kv: -kv[1][1])}
    return breakdown


if __name__ == "__main__":
    main()
