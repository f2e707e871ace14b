"""Benchmark of the fused FP8 block-scaled DeepSeek-V3 MoE layer on B200.

Default (N=1): BASELINE config 1, the DeepSeek-V3 decode layer (H=7168, I=2048, 32 local
experts of 256, top-8, ng8/kg4) at T=64 tokens -- the weight-bandwidth-bound regime the
metric quotes in "% HBM BW". One step = one call of the operator on one batch.
A sweep over configs 1, 2 and 4 (T = 1..8192, skewed routing) is attached as "sweep".

  value      tokens/s with inputs resident in HBM, CUDA events around each call,
             L2 flushed (256 MiB write, then read back) between timed calls
  e2e        tokens/s through the public API (fmoe_b200.kernel) with the activations
             copied from pinned host memory and the output copied back, every step, the
             copies overlapping the neighbouring steps' compute (serial_value: one step at
             a time)
  roofline   GEMM1 (the dominant kernel): algorithmic bytes per launch / its average
             duration (stage events recorded on the launch stream), against the measured
             HBM copy bandwidth in MEASURED_PEAKS.json
  cpu_baseline  the CPU oracle (PyTorch fp32 dequantise reference) on this host's cores,
             one call at the same workload

`--impl reference` times the reference operator (solution/cuda/kernel.cu, built from its
own source into oracle/_ref by oracle/build_ref.sh) on the same workload. The reference
has no CPU implementation of the path; its own code is CUDA, so it runs on the B200.

Multi-GPU (torchrun, N>1): BASELINE config 3, the full 256-expert layer under expert
parallelism (fmoe_b200.ep): rank r owns experts [r*256/N, (r+1)*256/N), holds 4096 tokens
(weak scaling), routes them, dispatches FP8 rows + scales + (expert, weight) pairs with an
NCCL all-to-all-v, runs the fused operator on what it received, and gets the partial
outputs back with a second all-to-all-v. The step time is the max over ranks (CUDA events,
all-reduce MAX); value counts the tokens of all ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "fused-moe-yws_b200"))
sys.path.insert(0, str(ROOT))

import fmoe_b200  # noqa: E402
from fmoe_b200 import workloads as W  # noqa: E402

FLOP_PER_ROW = 88_080_384          # 2*H*2I + 2*I*H for DS-V3
BYTES_PER_EXPERT = 44_050_944      # W13 + W2 FP8 + their fp32 block scales
GEMM1_BYTES_PER_EXPERT = 29_360_128 + 32 * 56 * 4
GEMM1_BYTES_PER_ROW = 7168 + 56 * 4 + 2 * 2048 + 16 * 4
GEMM1_FLOP_PER_ROW = 2 * 7168 * 2 * 2048
L2_FLUSH_BYTES = 256 << 20


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-f", self.path], stdout=subprocess.DEVNULL,
                stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        return False

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                if int(parts[0]) != self.gpu_index:
                    continue
                rows.append(parts)
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def make_workload(T: int, seed: int, skew: int = 0, device="cuda"):
    geo = W.DSV3
    acts = W.make_activations(geo, T, seed, device=device, skew_hot=skew)
    ws = W.make_weights(geo, seed, device=device)
    acts.update(ws)
    return acts


def routed_stats(inp):
    geo = W.DSV3
    idx, _ = fmoe_b200.route(inp["routing_logits"], inp["routing_bias"], geo.n_group,
                             geo.topk_group, geo.top_k, 2.5, num_local_experts=geo.num_local)
    local = idx[(idx >= 0) & (idx < geo.num_local)]
    rows = int(local.numel())
    active = int(torch.unique(local).numel())
    return rows, active


def layer_bytes(T, active):
    return active * BYTES_PER_EXPERT + T * (7168 + 224 + 1024) + T * 7168 * 2


def flush_l2(buf):
    """Evict L2 between timed calls: write a buffer twice L2's size, then read it back, so
    that the written lines are also written back to HBM here, outside the timed region (a
    preceding layer leaves L2 holding other data, not 126 MB of dirty lines)."""
    buf.zero_()
    buf.sum()


def time_device(inp, steps, warmup, flush, stage=False, tile_n=0):
    """Per-call device time (ms) with inputs resident; L2 flushed between calls."""
    args = W.operator_args(inp)
    out = torch.empty(args[0].shape[0], 7168, dtype=torch.bfloat16, device="cuda")
    for _ in range(warmup):
        fmoe_b200.kernel(*args, 0, 2.5, out=out, tile_n=tile_n)
    torch.cuda.synchronize()
    pairs, timers = [], []
    for _ in range(steps):
        flush_l2(flush)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        if stage:
            st = fmoe_b200.StageTimer()
            with st:
                e0.record()
                fmoe_b200.kernel(*args, 0, 2.5, out=out, tile_n=tile_n)
                e1.record()
            timers.append(st)
        else:
            e0.record()
            fmoe_b200.kernel(*args, 0, 2.5, out=out, tile_n=tile_n)
            e1.record()
        pairs.append((e0, e1))
    torch.cuda.synchronize()
    ms = [a.elapsed_time(b) for a, b in pairs]
    stages = [t.times_ms() for t in timers]
    return ms, stages, out


def time_graph(inp, steps, warmup, flush, tile_n=0):
    """Per-call device time (ms) of the operator replayed from a CUDA graph (all five
    kernels and the workspace memset captured once); L2 flushed between replays."""
    args = W.operator_args(inp)
    out = torch.empty(args[0].shape[0], 7168, dtype=torch.bfloat16, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(warmup):
            fmoe_b200.kernel(*args, 0, 2.5, out=out, tile_n=tile_n)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fmoe_b200.kernel(*args, 0, 2.5, out=out, tile_n=tile_n)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    pairs = []
    for _ in range(steps):
        flush_l2(flush)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        pairs.append((e0, e1))
    torch.cuda.synchronize()
    ms = [a.elapsed_time(b) for a, b in pairs]
    del graph
    return ms, out


def time_e2e(inp, steps, warmup):
    """Public API with host buffers, as a serving loop runs it: every step copies its
    activations from pinned host memory (H2D stream), calls fmoe_b200.kernel on the compute
    stream, and copies the bf16 result back (D2H stream). Two buffer slots let step i+1's
    upload and step i-1's download overlap step i's compute; every step's copies are inside
    the timed region. Returns (ms per step pipelined, ms per step serial, h2d, d2h bytes)."""
    names = ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale")
    T = inp["routing_logits"].shape[0]
    host = [{k: inp[k].cpu().pin_memory() for k in names} for _ in range(2)]
    dev = [{k: torch.empty_like(inp[k]) for k in names} for _ in range(2)]
    out_dev = [torch.empty(T, 7168, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    out_host = [torch.empty(T, 7168, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    h2d = sum(v.numel() * v.element_size() for v in host[0].values())
    d2h = out_host[0].numel() * 2
    comp = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    uploaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    downloaded = [torch.cuda.Event() for _ in range(2)]
    used = [False, False]

    def call(b):
        d = dev[b]
        fmoe_b200.kernel(d["routing_logits"], d["routing_bias"], d["hidden_states"],
                         d["hidden_states_scale"], inp["gemm1_weights"],
                         inp["gemm1_weights_scale"], inp["gemm2_weights"],
                         inp["gemm2_weights_scale"], 0, 2.5, out=out_dev[b])

    def step(i):
        b = i % 2
        with torch.cuda.stream(up):
            if used[b]:
                up.wait_event(computed[b])  # the slot's previous step has read its inputs
            for k in names:
                dev[b][k].copy_(host[b][k], non_blocking=True)
            uploaded[b].record(up)
        comp.wait_event(uploaded[b])
        if used[b]:
            comp.wait_event(downloaded[b])  # the slot's previous result has been read back
        call(b)
        computed[b].record(comp)
        with torch.cuda.stream(down):
            down.wait_event(computed[b])
            out_host[b].copy_(out_dev[b], non_blocking=True)
            downloaded[b].record(down)
        used[b] = True

    def run(n, pipelined):
        for i in range(n):
            step(i)
            if not pipelined:  # the next upload starts after this step's result is back
                up.wait_event(downloaded[i % 2])

    run(warmup, True)
    torch.cuda.synchronize()
    res = []
    for pipelined in (True, False):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(comp)
        up.wait_stream(comp)
        down.wait_stream(comp)
        run(steps, pipelined)
        comp.wait_stream(down)
        e1.record(comp)
        torch.cuda.synchronize()
        res.append(e0.elapsed_time(e1) / steps)
    return res[0], res[1], h2d, d2h


def cpu_baseline(T, seed, skew=0):
    """CPU oracle on this host's cores, one call of the same workload (bounded sample)."""
    import oracle

    torch.set_num_threads(os.cpu_count() or 1)
    geo = W.DSV3
    inp = make_workload(T, seed, skew, device="cpu")
    t0 = time.perf_counter()
    oracle.moe_forward(*W.operator_args(inp), 0, 2.5, geo.n_group, geo.topk_group, geo.top_k)
    dt = time.perf_counter() - t0
    return {"value": T / dt, "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"one call of the T={T} DS-V3 layer (dequantise + fp32 GEMMs), {dt:.2f} s"}


def sweep(seed, hbm_peak, fp8_peak, tiles=(0,), tokens=None):
    """Configs 1, 2 and 4 over T; `tiles` lists the token tiles timed per case (0 = the
    autotune table). Tiles above 16 are skipped for T < 64 and 128 for T < 512. `tokens`
    replaces the cases by uniform-routing ones at those token counts."""
    res = []
    lib = fmoe_b200.load_library()
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    cases = [("config1", 1, 0), ("config1", 4, 0), ("config1", 16, 0), ("config1", 64, 0),
             ("config2", 512, 0), ("config2", 2048, 0), ("config2", 4096, 0),
             ("config2", 8192, 0), ("config4", 4096, 8)]
    if tokens:
        cases = [("config1" if T <= 64 else "config2", T, 0) for T in tokens]
    for cfg, T, skew in cases:
        inp = make_workload(T, seed, skew)
        rows, active = routed_stats(inp)
        b = layer_bytes(T, active)
        for tile in tiles:
            if (tile > 16 and T < 64) or (tile == 128 and T < 512):
                continue
            ms_e, stages, _ = time_device(inp, steps=10, warmup=3, flush=flush, stage=True,
                                          tile_n=tile)
            ms, _ = time_graph(inp, steps=10, warmup=3, flush=flush, tile_n=tile)
            t = statistics.median(ms)
            st = [statistics.median(s[i] for s in stages) for i in range(5)]
            res.append({"config": cfg, "T": T, "skew_hot": skew, "rows": rows,
                        "active_experts": active,
                        "tile_n": tile or lib.fmoe_autotune_tile_n(T),
                        "us_per_call": round(t * 1e3, 1),
                        "us_per_call_eager": round(statistics.median(ms_e) * 1e3, 1),
                        "tokens_per_s": round(T / (t * 1e-3), 1),
                        "hbm_gbs": round(b / (t * 1e-3) / 1e9, 1),
                        "hbm_frac": round(b / (t * 1e-3) / 1e9 / hbm_peak, 3),
                        "fp8_tflops": round(rows * FLOP_PER_ROW / (t * 1e-3) / 1e12, 1),
                        "fp8_frac": round(rows * FLOP_PER_ROW / (t * 1e-3) / 1e12 / fp8_peak,
                                          3),
                        "stage_us": dict(zip(fmoe_b200.StageTimer.STAGES,
                                             [round(x * 1e3, 1) for x in st]))})
        del inp
        torch.cuda.empty_cache()
    return res


def run_ep(args, world, rank, local):
    """Config 3: the 256-expert layer under expert parallelism over `world` ranks."""
    from fmoe_b200 import ep

    geo = W.DSV3
    T = args.tokens if args.tokens_set else 4096
    per = 256 // world
    weights = W.make_expert_slice(geo, args.seed, rank * per, per, device="cuda")
    acts = W.make_activations(geo, T, args.seed + 1009 * rank, device="cuda")
    layer = ep.ExpertParallelMoE(weights=weights, exchange=args.exchange)
    a4 = [acts[k] for k in W.OPERATOR_ARGS[:4]]
    for _ in range(args.warmup):
        layer.forward(*a4)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    gpu_index = local
    pairs = []
    with ClockSampler(gpu_index) as clk:
        for _ in range(args.steps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            layer.forward(*a4)
            e1.record()
            pairs.append((e0, e1))
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
    total = torch.tensor([sum(x.elapsed_time(y) for x, y in pairs)], device="cuda")
    dist.all_reduce(total, op=dist.ReduceOp.MAX)
    ms_per_step = float(total.item()) / args.steps
    # stage breakdown (one extra timed pass, outside the measured steps)
    layer.forward(*a4, timed=True)
    tm = layer.timings
    br = torch.tensor([tm.route_ms, tm.dispatch_ms, tm.compute_ms, tm.combine_ms], device="cuda")
    dist.all_reduce(br, op=dist.ReduceOp.MAX)
    # e2e: activations from pinned host memory, output back to the host, every step
    names = W.OPERATOR_ARGS[:4]
    host = {k: acts[k].cpu().pin_memory() for k in names}
    dev = {k: torch.empty_like(acts[k]) for k in names}
    out_host = torch.empty(T, geo.hidden, dtype=torch.bfloat16).pin_memory()
    e2e_pairs = []
    for i in range(args.steps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for k in names:
            dev[k].copy_(host[k], non_blocking=True)
        o = layer.forward(*[dev[k] for k in names])
        out_host.copy_(o, non_blocking=True)
        e1.record()
        e2e_pairs.append((e0, e1))
    torch.cuda.synchronize()
    e2e_t = torch.tensor([sum(x.elapsed_time(y) for x, y in e2e_pairs)], device="cuda")
    dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_t.item()) / args.steps
    h2d = sum(host[k].numel() * host[k].element_size() for k in names)
    rows = torch.tensor([0], device="cuda")
    line = {
        "metric": "MoE layer tokens/s (DS-V3 full 256-expert layer, expert parallel)",
        "value": round(world * T / (ms_per_step * 1e-3), 1), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3 x e4m3 -> fp32 (tcgen05 kind::f8f6f4), fp32 block-scale promotion",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights, FP8 128-block scales)",
        "config": {"workload": "config3_dsv3_ep", "tokens_per_rank": T, "hidden": 7168,
                   "intermediate": 2048, "experts": 256, "experts_per_rank": per, "top_k": 8,
                   "n_group": 8, "topk_group": 4, "parallelism": f"ep{world}",
                   "collectives": ("rows stored into the peers' buffers over NVLink (CUDA IPC), "
                                   "counts all-gather and one-element all-reduce barriers (NCCL)"
                                   if args.exchange == "p2p" else
                                   "NCCL all-to-all-v dispatch + combine, counts all-to-all"),
                   "l2": f"weights {per * 44.05 / 1000:.1f} GB per rank > L2"},
        "breakdown_ms_max_over_ranks": {"route": round(float(br[0]), 3),
                                        "dispatch": round(float(br[1]), 3),
                                        "compute": round(float(br[2]), 3),
                                        "combine": round(float(br[3]), 3)},
        "clocks": clk.summary(),
        "e2e": {"value": round(world * T / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": T * geo.hidden * 2},
        # routing, send plan, pack, unpack, the operator's 5 kernels, (P2P: return), combine
        "gpu_launches": (10 + (args.exchange == "p2p")) * args.steps,
    }
    layer.close()
    return line


def run_reference(args, rank):
    so = ROOT / "oracle" / "_ref" / "ref_kernel.so"
    base = {"metric": "MoE layer tokens/s (DS-V3 decode, T=64)", "impl": "reference"}
    if rank != 0:
        return None
    if not so.exists():
        base["unavailable"] = "reference kernel not built (oracle/build_ref.sh needs the source)"
        return base
    import tvm_ffi

    kern = tvm_ffi.load_module(str(so))["kernel"]
    T = args.tokens
    inp = make_workload(T, args.seed)
    a = W.operator_args(inp)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    for _ in range(args.warmup):
        kern(*a, 0, 2.5)
    torch.cuda.synchronize()
    pairs = []
    for _ in range(args.steps):
        flush_l2(flush)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        kern(*a, 0, 2.5)
        e1.record()
        pairs.append((e0, e1))
    torch.cuda.synchronize()
    ms = [x.elapsed_time(y) for x, y in pairs]
    t = sum(ms) / len(ms)
    v = T / (t * 1e-3)
    base.update({
        "value": v, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3 x e4m3 -> fp32 (reference: fp32 SIMT / f16, tf32-class mma.sync)",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights, FP8 128-block scales)",
        "config": {"workload": f"config1_dsv3_decode_T{T}", "tokens": T, "hidden": 7168,
                   "intermediate": 2048, "experts": 256, "local_experts": 32, "top_k": 8,
                   "l2": "flushed between calls (256 MiB write, then read back)"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": 1, "kind": "reference",
                         "sample": "reference solution/cuda/kernel.cu (its own CUDA code; it has "
                                   "no CPU implementation) timed on the B200, one host thread"},
    })
    return base


# The JSON line is the only thing this script writes to stdout. Libraries loaded later
# (NCCL prints its version there, for one) write to the process's file descriptor 1 from
# C, so descriptor 1 is pointed at stderr and the result goes to a duplicate of the
# original stdout.
_RESULT_OUT = None


def _claim_stdout():
    global _RESULT_OUT
    if _RESULT_OUT is None:
        sys.stdout.flush()
        _RESULT_OUT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)


def emit(line: dict) -> None:
    _RESULT_OUT.write(json.dumps(line) + "\n")
    _RESULT_OUT.flush()


def main():
    _claim_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--skew", type=int, default=0,
                    help="route every token onto this many hot local experts (config 4: 8); "
                         "0 = grouped top-k over random logits")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--exchange", choices=("p2p", "nccl"), default="p2p",
                    help="expert-parallel runs (N > 1): rows over peer memory or NCCL all-to-all")
    ap.add_argument("--sweep-tiles", default="0",
                    help="comma-separated token tiles timed per sweep case (0 = autotune)")
    ap.add_argument("--sweep-tokens", default="",
                    help="comma-separated token counts replacing the sweep's cases")
    args = ap.parse_args()
    args.tokens_set = args.tokens is not None
    if args.tokens is None:
        args.tokens = 64
    assert args.warmup >= 3, "at least 3 warm-up steps"

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=120))

    if args.impl == "reference":
        line = run_reference(args, rank)
        if line is not None:
            emit(line)
        if world > 1:
            dist.destroy_process_group()
        return

    if world > 1:
        line = run_ep(args, world, rank, local)
        if rank == 0:
            emit(line)
        dist.barrier()
        dist.destroy_process_group()
        return

    hbm_peak, bf16_peak, peak_src = load_peaks()
    fp8_peak = 2.0 * bf16_peak
    T = args.tokens
    inp = make_workload(T, args.seed, args.skew)
    rows, active = routed_stats(inp)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    fmoe_b200.kernel(*W.operator_args(inp), 0, 2.5)  # first call: library setup
    torch.cuda.synchronize()

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    gpu_index = int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local]) \
        if os.environ.get("CUDA_VISIBLE_DEVICES") else local
    # eager pass with stage events (per-kernel durations for the roofline)
    ms_eager, stages, _ = time_device(inp, args.steps, args.warmup, flush, stage=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(gpu_index) as clk:
        ms, _ = time_graph(inp, args.steps, args.warmup, flush)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
    clocks = clk.summary()
    total_ms = sum(ms)
    if world > 1:
        t = torch.tensor([total_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = world * T / (ms_per_step * 1e-3)

    g1 = [s[2] for s in stages]
    g1_ms = sum(g1) / len(g1)
    g1_bytes = active * GEMM1_BYTES_PER_EXPERT + rows * GEMM1_BYTES_PER_ROW
    achieved = g1_bytes / (g1_ms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "kernel": "grouped_gemm_kernel<GEMM1+SwiGLU>",
                "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(achieved / hbm_peak, 3), "peak_source": peak_src,
                "traffic": None, "bytes_per_launch": g1_bytes,
                "stage_us": dict(zip(fmoe_b200.StageTimer.STAGES,
                                     [round(sum(s[i] for s in stages) / len(stages) * 1e3, 1)
                                      for i in range(5)])),
                "layer_hbm_frac": round(layer_bytes(T, active) / (ms_per_step * 1e-3) / 1e9
                                        / hbm_peak, 3)}
    tile_n = fmoe_b200.load_library().fmoe_autotune_tile_n(T)
    if args.skew:
        # compute-bound case: GEMM1 against the FP8 dense peak
        g1_flops = rows * GEMM1_FLOP_PER_ROW
        tf = g1_flops / (g1_ms * 1e-3) / 1e12
        roofline.update({"bound": "tensor", "achieved": round(tf, 1), "peak": fp8_peak,
                         "unit": "TFLOP/s", "frac": round(tf / fp8_peak, 3),
                         "peak_source": peak_src + ", fp8 = 2 x bf16",
                         "flops_per_launch": g1_flops})
        roofline.pop("bytes_per_launch")
    if tile_n == 128:
        roofline["kernel"] = "grouped_gemm_tm_kernel<GEMM1+SwiGLU>"
    traffic_file = ROOT / "profiles" / "traffic.json"
    if traffic_file.exists():
        key = f"gemm1_T{T}" + (f"_hot{args.skew}" if args.skew else "")
        tr = json.loads(traffic_file.read_text()).get(key)
        if tr:
            roofline["traffic"] = tr

    e2e_ms, e2e_serial_ms, h2d, d2h = time_e2e(inp, args.steps, args.warmup)
    e2e = {"value": round(T / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
           "mode": "copies on separate H2D / D2H streams, overlapping the neighbouring "
                   "steps' compute (2 buffer slots)",
           "serial_value": round(T / (e2e_serial_ms * 1e-3), 1)}

    line = {
        "metric": (f"MoE layer tokens/s (DS-V3 decode, T={T})" if not args.skew else
                   f"MoE layer tokens/s (DS-V3, T={T}, {args.skew} hot experts)"),
        "value": round(value, 1),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4), "us_per_call": round(ms_per_step * 1e3, 1),
        "us_per_call_eager": round(statistics.mean(ms_eager) * 1e3, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3 x e4m3 -> fp32 (tcgen05 kind::f8f6f4), fp32 block-scale promotion",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights, FP8 128-block scales)",
        "config": {"workload": (f"config1_dsv3_decode_T{T}" if not args.skew else
                                f"config4_dsv3_T{T}_hot{args.skew}"), "tokens_per_rank": T,
                   "hidden": 7168, "intermediate": 2048, "experts": 256, "local_experts": 32,
                   "top_k": 8, "n_group": 8, "topk_group": 4, "routed_rows": rows,
                   "active_experts": active, "tile_n": tile_n,
                   "parallelism": f"replicas x{world}",
                   "l2": "flushed between calls (256 MiB write, then read back); weights > L2",
                   "launch": "one CUDA graph replay per step (memset + 5 PDL kernels)"},
        "roofline": roofline, "clocks": clocks, "e2e": e2e,
        "gpu_launches": 5 * args.steps,
    }
    if rank == 0:
        if not args.no_cpu and world == 1:
            line["cpu_baseline"] = cpu_baseline(T, args.seed, args.skew)
        if not args.no_sweep and world == 1:
            line["sweep"] = sweep(args.seed, hbm_peak, fp8_peak,
                                  tiles=tuple(int(x) for x in args.sweep_tiles.split(",")),
                                  tokens=[int(x) for x in args.sweep_tokens.split(",") if x])
            line["sweep_fp8_peak_tflops"] = fp8_peak
        emit(line)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
