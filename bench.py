"""Benchmark of the fused FP8 block-scaled DeepSeek-V3 MoE layer on B200.

Headline, at every N (1, 2, 4, 8 GPUs, one process per GPU): BASELINE config 3, the full
256-expert DeepSeek-V3 layer (H=7168, I=2048, top-8, ng8/kg4) with 4096 tokens per rank
(weak scaling). At N=1 the one GPU holds all 256 experts and runs the operator once per
step (E_local = 256, `fmoe_b200.kernel`); at N>1 rank r owns experts [r*256/N, (r+1)*256/N)
and the layer runs under expert parallelism (`fmoe_b200.ep`): route, dispatch the tokens'
FP8 rows + scales + (expert, weight) pairs to the owning ranks over NVLink, compute, return
the partial outputs, combine. One step = one pass of the layer over every rank's 4096
tokens; the step time is the max over ranks (CUDA events), `value` counts all ranks' tokens.

  value      tokens/s with inputs resident in HBM (weights 11.3 GB / N per rank > L2; L2 is
             also flushed between steps at N=1)
  e2e        tokens/s through the public API with each step's activations copied from pinned
             host memory and the bf16 output copied back, inside the timed region, copies
             overlapping neighbouring steps over two buffer slots
  roofline   the dominant kernel (GEMM1+SwiGLU): algorithmic bytes or FLOPs per launch / its
             duration (CUDA events on the launch stream), against MEASURED_PEAKS.json's HBM
             copy bandwidth or the FP8 dense rate measured live by fmoe_probe_fp8_mma_rate;
             the bound is whichever roofline time is longer
  ep_parity  32 tokens per rank of the step's output against the single-GPU operator run
             on each rank's experts (local_expert_offset) and summed in rank order
  placement  (N>1) which experts each rank owns, from a calibration batch of other
             tokens: by default the contiguous slices refined by cost-lowering expert swaps
             (--placement local); --placement balanced (greedy on 128-row tile counts) or
             contiguous (the reference's 256/N slices) for comparison
  cpu_baseline  (N=1) the CPU oracle (PyTorch fp32 dequantise reference) on this host's
             cores, a bounded sample: 64 tokens of the same layer
  sweep      (N=1) BASELINE configs 1, 2 and 4 on one 32-expert slice (T = 1..8192 and the
             skewed case), each with its own roofline

`--impl reference` runs the reference operator (solution/cuda/kernel.cu, built from its own
source into oracle/_ref by oracle/build_ref.sh) on the same workload at every N: each rank
holds all 256 experts and calls the reference once per 32-expert slice
(local_expert_offset = 32 s, s = 0..7), summing the eight bf16 slice outputs in fp32 and
casting to bf16 -- the reference computes one slice per call and leaves the sum over slices
to its caller (kernel.cu:538-545). Its implementation of the path is CUDA only, so it runs
on the B200; at N=1 it also times its own operator on the sweep's cases.

`--workload slice` times one 32-expert slice (`--tokens`, `--skew`) instead, for profiles.
"""
from __future__ import annotations

import argparse
import datetime
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

H, I = 7168, 2048
FLOP_PER_ROW = 88_080_384          # 2*H*2I + 2*I*H for DS-V3
GEMM1_FLOP_PER_ROW = 2 * H * 2 * I
GEMM2_FLOP_PER_ROW = 2 * I * H
BYTES_PER_EXPERT = 44_050_944      # W13 + W2 FP8 + their fp32 block scales
GEMM1_BYTES_PER_EXPERT = 29_360_128 + 32 * 56 * 4
GEMM2_BYTES_PER_EXPERT = 14_680_064 + 56 * 16 * 4
GEMM1_BYTES_PER_ROW = 7168 + 56 * 4 + 2 * 2048 + 16 * 4   # FP8 row + scales in, hi/lo C out
GEMM2_BYTES_PER_ROW = 2 * 2048 + 16 * 4 + 7168 * 2         # hi/lo C + scales in, bf16 row out
L2_FLUSH_BYTES = 256 << 20
LAYER_TOKENS = 4096
PARITY_TOKENS = 32
CAL_SEED = 7777  # seed offset of the expert-placement calibration batch (N > 1)
CPU_SAMPLE_TOKENS = 64
RSF = 2.5


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def measure_fp8_peak():
    """Dense FP8 tensor-core rate of this GPU, measured now (tcgen05 kind::f8f6f4
    M128 x N256 x K32 back to back on every SM)."""
    best = max(fmoe_b200.probe_fp8_mma_rate(16384)["tflops"] for _ in range(3))
    return best


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


def gpu_index_of(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    return int(vis.split(",")[local]) if vis else local


# ---------------------------------------------------------------------------- workloads
def layer_activations(seed: int, rank: int, T: int, device="cuda"):
    """Rank `rank`'s tokens of the config-3 layer. The routing bias is a layer parameter,
    the same on every rank (drawn from the base seed); the tokens differ per rank."""
    acts = W.make_activations(W.DSV3, T, seed + 1009 * rank, device=device)
    acts["routing_bias"] = W.make_activations(W.DSV3, 1, seed, device=device)["routing_bias"]
    return acts


def layer_weights(seed: int, first: int, count: int, device="cuda"):
    """Experts [first, first + count) of the 256-expert layer; expert e's values do not
    depend on which slice holds it (one generator per (seed, expert))."""
    return W.make_expert_slice(W.DSV3, seed, first, count, device=device)


def layer_config(T: int, world: int, exchange: str, placement: str = "local",
                 host_sync: bool = False) -> dict:
    per = 256 // world
    cfg = {"workload": "config3_dsv3_full_layer", "tokens_per_rank": T, "hidden": H,
           "intermediate": I, "experts": 256, "experts_per_rank": per, "top_k": 8,
           "n_group": 8, "topk_group": 4, "routed_scaling_factor": RSF,
           "parallelism": f"ep{world}" if world > 1 else "single GPU, all 256 experts local",
           "l2": f"weights {per * BYTES_PER_EXPERT / 1e9:.1f} GB per rank > L2 (126 MB)"}
    if world > 1:
        cfg["collectives"] = (
            "rows stored into the peers' buffers over NVLink (CUDA IPC), counts all-gather and "
            "one-element all-reduce barriers (NCCL); " + (
                "counts read on the host each step" if host_sync else
                "row offsets and received-row counts computed on the device (no host round "
                "trip per step)") if exchange == "p2p" else
            "NCCL all-to-all-v dispatch + combine, counts all-to-all")
        cfg["placement"] = {
            "balanced": "balanced: experts assigned to ranks by longest-processing-time greedy "
                        "on their 128-row tile counts in a calibration batch (other tokens, "
                        "same layer)",
            "local": "local: contiguous slices refined by expert swaps that lower the largest "
                     "rank cost (128-row tiles + received tokens) on a calibration batch "
                     "(other tokens, same layer)",
        }.get(placement, "contiguous 256/N-expert slices")
    return cfg


def routed_stats(acts, first: int, count: int):
    idx, _ = fmoe_b200.route(acts["routing_logits"], acts["routing_bias"], 8, 4, 8, RSF,
                             num_local_experts=count, local_expert_offset=first)
    local = idx[(idx >= first) & (idx < first + count)]
    return int(local.numel()), int(torch.unique(local).numel())


def flush_l2(buf):
    """Evict L2 between timed calls: write a buffer twice L2's size, then read it back, so
    that the written lines are also written back to HBM here, outside the timed region."""
    buf.zero_()
    buf.sum()


# ---------------------------------------------------------------------------- rooflines
def roofline(kernel: str, nbytes: float, flops: float, ms: float, hbm: float, fp8: float,
             fp8_src: str, hbm_src: str) -> dict:
    """The bound is whichever roofline time (bytes / HBM bandwidth, FLOPs / FP8 rate) is
    longer; achieved = algorithmic bytes or FLOPs of one launch / its duration."""
    t_hbm = nbytes / (hbm * 1e9)
    t_tc = flops / (fp8 * 1e12)
    s = ms * 1e-3
    if t_hbm >= t_tc:
        ach, peak, unit, bound, src = nbytes / s / 1e9, hbm, "GB/s", "hbm", hbm_src
    else:
        ach, peak, unit, bound, src = flops / s / 1e12, fp8, "TFLOP/s", "tensor", fp8_src
    return {"bound": bound, "kernel": kernel, "achieved": round(ach, 1), "peak": round(peak, 1),
            "unit": unit, "frac": round(ach / peak, 3), "peak_source": src,
            "bytes_per_launch": int(nbytes), "flops_per_launch": int(flops),
            "us": round(ms * 1e3, 1),
            "hbm_frac": round(nbytes / s / 1e9 / hbm, 3),
            "fp8_frac": round(flops / s / 1e12 / fp8, 3)}


def layer_bytes(T, active):
    return active * BYTES_PER_EXPERT + T * (7168 + 224 + 1024) + T * 7168 * 2


def kernel_rooflines(rows, active, stage_ms, hbm, fp8, fp8_src, hbm_src, tile_n):
    fam = "grouped_gemm_tm_kernel" if tile_n == 128 else "grouped_gemm_kernel"
    g1 = roofline(f"{fam}<GEMM1+SwiGLU>",
                  active * GEMM1_BYTES_PER_EXPERT + rows * GEMM1_BYTES_PER_ROW,
                  rows * GEMM1_FLOP_PER_ROW, stage_ms[2], hbm, fp8, fp8_src, hbm_src)
    g2 = roofline(f"{fam}<GEMM2>", active * GEMM2_BYTES_PER_EXPERT + rows * GEMM2_BYTES_PER_ROW,
                  rows * GEMM2_FLOP_PER_ROW, stage_ms[3], hbm, fp8, fp8_src, hbm_src)
    return g1, g2


def stored_traffic(key: str):
    """DRAM bytes of one GEMM1 launch from an ncu capture of this workload (profiles/)."""
    f = ROOT / "profiles" / "traffic.json"
    if f.exists():
        return json.loads(f.read_text()).get(key)
    return None


# ---------------------------------------------------------------------------- timing
def time_graph(fn, steps, warmup, flush):
    """Device time (ms) of each of `steps` replays of `fn` captured in one CUDA graph, L2
    flushed before each replay."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
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
    return ms


def time_stages(fn, steps, flush):
    """Eager calls with stage events (route, permute, gemm1, gemm2, combine), per-stage
    median in ms, and the per-call times."""
    res, tot = [], []
    for _ in range(steps):
        flush_l2(flush)
        st = fmoe_b200.StageTimer()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with st:
            e0.record()
            fn()
            e1.record()
        torch.cuda.synchronize()
        res.append(st.times_ms())
        tot.append(e0.elapsed_time(e1))
    return [statistics.median(r[i] for r in res) for i in range(5)], tot


def time_e2e(acts, weights, steps, warmup, call):
    """Public API with host buffers, as a serving loop runs it: every step copies its
    activations from pinned host memory (H2D stream), runs `call` on the compute stream,
    and copies the bf16 result back (D2H stream). Two buffer slots let step i+1's upload
    and step i-1's download overlap step i's compute; every step's copies are inside the
    timed region. Returns (ms per step pipelined, ms per step serial, h2d, d2h bytes)."""
    names = W.OPERATOR_ARGS[:4]
    T = acts["routing_logits"].shape[0]
    host = [{k: acts[k].cpu().pin_memory() for k in names} for _ in range(2)]
    dev = [{k: torch.empty_like(acts[k]) for k in names} for _ in range(2)]
    out_dev = [torch.empty(T, H, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    out_host = [torch.empty(T, H, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    h2d = sum(v.numel() * v.element_size() for v in host[0].values())
    d2h = out_host[0].numel() * 2
    comp = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    uploaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    downloaded = [torch.cuda.Event() for _ in range(2)]
    used = [False, False]

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
        r = call(*[dev[b][k] for k in names], out=out_dev[b])
        if r.data_ptr() != out_dev[b].data_ptr():
            out_dev[b].copy_(r)
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
        if dist.is_initialized():
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(comp)
        up.wait_stream(comp)
        down.wait_stream(comp)
        run(steps, pipelined)
        comp.wait_stream(down)
        e1.record(comp)
        torch.cuda.synchronize()
        res.append(max_over_ranks(e0.elapsed_time(e1)) / steps)
    return res[0], res[1], h2d, d2h


def max_over_ranks(x: float) -> float:
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------- checks
def ep_parity(out, acts, weights, world, rank, per, layer=None):
    """The step's output for this rank's first PARITY_TOKENS tokens against the
    single-GPU operator: every rank runs the operator on all ranks' sampled tokens with its
    own experts (`fmoe_b200.kernel` with local_expert_offset = rank * per for contiguous
    slices; under a placement, the routing kernel, the ids mapped to placement positions
    and `fmoe_b200.forward_routed` on the rank's experts), the partials are summed in fp32
    in rank order and rounded to bf16. Tolerance atol = rtol = 2e-2 (bf16 output)."""
    n = PARITY_TOKENS
    names = W.OPERATOR_ARGS[:4]
    mine = {"routing_logits": acts["routing_logits"][:n].contiguous(),
            "routing_bias": acts["routing_bias"],
            "hidden_states": acts["hidden_states"][:n].contiguous(),
            "hidden_states_scale": acts["hidden_states_scale"][:, :n].contiguous()}
    if world > 1:
        lg = torch.empty(world * n, 256, dtype=torch.float32, device="cuda")
        dist.all_gather_into_tensor(lg, mine["routing_logits"])
        hs = torch.empty(world * n, H, dtype=torch.uint8, device="cuda")
        dist.all_gather_into_tensor(hs, mine["hidden_states"].view(torch.uint8))
        sc = torch.empty(world * (H // 128), n, dtype=torch.float32, device="cuda")
        dist.all_gather_into_tensor(sc, mine["hidden_states_scale"])
        sc = sc.view(world, H // 128, n).permute(1, 0, 2).reshape(H // 128, world * n)
        allin = {"routing_logits": lg, "routing_bias": mine["routing_bias"],
                 "hidden_states": hs.view(torch.float8_e4m3fn),
                 "hidden_states_scale": sc.contiguous()}
    else:
        allin = mine
    wts = [weights[k] for k in W.OPERATOR_ARGS[4:]]
    if layer is not None and layer.placement is not None:
        idx, w = fmoe_b200.route(allin["routing_logits"], allin["routing_bias"], 8, 4, 8, RSF)
        part = fmoe_b200.forward_routed(layer.place_ids(idx).contiguous(), w,
                                        allin["hidden_states"], allin["hidden_states_scale"],
                                        *wts, rank * per, 256)
    else:
        part = fmoe_b200.kernel(*[allin[k] for k in names], *wts, rank * per, RSF)
    if world > 1:
        parts = torch.empty(world, world * n, H, dtype=torch.bfloat16, device="cuda")
        dist.all_gather_into_tensor(parts, part)
        acc = torch.zeros(n, H, dtype=torch.float32, device="cuda")
        for r in range(world):  # rank order, as the layer's combine
            acc += parts[r, rank * n:(rank + 1) * n].float()
        ref = acc.to(torch.bfloat16)
    else:
        ref = part
    got = out[:n].float()
    ref = ref.float()
    diff = (got - ref).abs()
    excess = float((diff - (2e-2 + 2e-2 * ref.abs())).max())
    rel = float(diff.norm() / ref.norm().clamp_min(1e-12))
    stats = torch.tensor([float(diff.max()), rel, excess], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    return {"tokens_checked": n * world, "max_abs": round(float(stats[0]), 6),
            "rel_rms": round(float(stats[1]), 6), "ok": bool(stats[2] <= 0.0),
            "tolerance": "atol 2e-2 + rtol 2e-2 on the bf16 output",
            "reference": ("single-GPU operator on each rank's experts, summed in rank "
                          "order" if world > 1 else
                          "single-GPU operator on the sampled tokens alone")}


def cpu_baseline_layer(acts, weights):
    """CPU oracle on this host's cores: the first CPU_SAMPLE_TOKENS tokens of the layer
    (all 256 experts; only routed experts are dequantised, one at a time)."""
    import oracle

    torch.set_num_threads(os.cpu_count() or 1)
    n = CPU_SAMPLE_TOKENS
    a = [acts["routing_logits"][:n].cpu(), acts["routing_bias"].cpu(),
         acts["hidden_states"][:n].cpu(), acts["hidden_states_scale"][:, :n].cpu()]
    t0 = time.perf_counter()
    oracle.moe_forward(*a, *[weights[k] for k in W.OPERATOR_ARGS[4:]], 0, RSF, 8, 4, 8)
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 2), "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": (f"{n} tokens of the config-3 layer (all 256 experts; dequantise + fp32 "
                       f"GEMMs of the routed experts), {dt:.1f} s")}


# ---------------------------------------------------------------------------- our arm
def run_layer_single(args, peaks, flush):
    """N=1: the whole 256-expert layer on one GPU, one operator call per step."""
    hbm, fp8, hbm_src, fp8_src = peaks
    T = args.tokens or LAYER_TOKENS
    weights = layer_weights(args.seed, 0, 256)
    acts = layer_activations(args.seed, 0, T)
    rows, active = routed_stats(acts, 0, 256)
    wargs = [weights[k] for k in W.OPERATOR_ARGS[4:]]
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")

    def call(*a4, out=out):
        return fmoe_b200.kernel(*a4, *wargs, 0, RSF, out=out)

    a4 = [acts[k] for k in W.OPERATOR_ARGS[:4]]
    call(*a4)
    torch.cuda.synchronize()
    stage_ms, eager_ms = time_stages(lambda: call(*a4), args.steps, flush)
    with ClockSampler(gpu_index_of(0)) as clk:
        ms = time_graph(lambda: call(*a4), args.steps, args.warmup, flush)
        torch.cuda.synchronize()
    ms_per_step = sum(ms) / len(ms)
    tile_n = fmoe_b200.tile_n(fmoe_b200.make_problem(T, 256, 256, H, I))
    g1, g2 = kernel_rooflines(rows, active, stage_ms, hbm, fp8, fp8_src, hbm_src, tile_n)
    g1["traffic"] = stored_traffic(f"gemm1_layer_T{T}")
    g1["traffic_source"] = "ncu dram__bytes_read.sum + dram__bytes_write.sum (profiles/)"
    g1["stage_us"] = dict(zip(fmoe_b200.StageTimer.STAGES, [round(x * 1e3, 1) for x in stage_ms]))
    g1["gemm2"] = g2
    g1["layer"] = roofline("whole layer (5 kernels)", layer_bytes(T, active), rows * FLOP_PER_ROW,
                           ms_per_step, hbm, fp8, fp8_src, hbm_src)
    out_ref = call(*a4).clone()
    parity = ep_parity(out_ref, acts, weights, 1, 0, 256)
    e2e_ms, e2e_serial, h2d, d2h = time_e2e(acts, weights, args.steps, args.warmup, call)
    line = base_line(args, 1, T, ms_per_step, layer_config(T, 1, args.exchange))
    line["config"].update({"routed_rows": rows, "active_experts": active, "tile_n": tile_n,
                           "launch": "one operator call per step (library graph cache: one "
                                     "CUDA graph replay of memset + 5 PDL kernels)",
                           "l2_flush": "256 MiB written and read back between steps"})
    line.update({"us_per_call_eager": round(statistics.median(eager_ms) * 1e3, 1),
                 "roofline": g1, "clocks": clk.summary(), "ep_parity": parity,
                 "e2e": {"value": round(T / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                         "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                         "mode": "copies on separate H2D / D2H streams, overlapping the "
                                 "neighbouring steps' compute (2 buffer slots)",
                         "serial_value": round(T / (e2e_serial * 1e-3), 1)},
                 "gpu_launches": 5 * args.steps})
    if not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline_layer(acts, weights)
    del acts
    if not args.no_sweep:
        w32 = {k: v[:32] for k, v in weights.items()}
        line["sweep"] = sweep_ours(args, w32, peaks, flush)
        line["sweep_peaks"] = {"hbm_gbs": hbm, "hbm_source": hbm_src, "fp8_tflops": round(fp8, 1),
                               "fp8_source": fp8_src}
    return line


def run_ep(args, world, rank, local, peaks):
    """N>1: the 256-expert layer under expert parallelism over `world` ranks."""
    from fmoe_b200 import ep

    hbm, fp8, hbm_src, fp8_src = peaks
    T = args.tokens or LAYER_TOKENS
    per = 256 // world
    acts = layer_activations(args.seed, rank, T)
    placement = None
    if args.placement != "contiguous":
        # expert loads of a calibration batch: other tokens (seed offset), the same layer
        cal = W.make_activations(W.DSV3, T, args.seed + CAL_SEED + 1009 * rank, device="cuda")
        placement = ep.calibrate_placement(
            lambda lg, b: fmoe_b200.route(lg, b, 8, 4, 8, RSF), cal["routing_logits"],
            acts["routing_bias"], 256, mode=args.placement, search=args.placement_search)
        del cal
    mine = placement[rank * per:(rank + 1) * per] if placement else range(rank * per,
                                                                          (rank + 1) * per)
    weights = W.make_expert_set(W.DSV3, args.seed, mine, device="cuda")
    layer = ep.ExpertParallelMoE(weights=weights, exchange=args.exchange, placement=placement,
                                 max_tokens=None if args.ep_host_sync else T,
                                 fused_return=not args.ep_separate_return)
    a4 = [acts[k] for k in W.OPERATOR_ARGS[:4]]
    for _ in range(args.warmup):
        layer.forward(*a4)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    pairs = []
    with ClockSampler(gpu_index_of(local)) as clk:
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
    ms_per_step = max_over_ranks(sum(x.elapsed_time(y) for x, y in pairs)) / args.steps
    # stage breakdown and the local operator's kernel stages (extra passes outside the timed
    # steps; the first one goes through the stage-timed path for the first time, so the
    # second one is kept)
    for _ in range(2):
        dist.barrier()
        torch.cuda.synchronize()
        out = layer.forward(*a4, timed=True)
    tm = layer.timings
    br = torch.tensor([tm.route_ms, tm.dispatch_ms, tm.compute_ms, tm.combine_ms],
                      device="cuda")
    dist.all_reduce(br, op=dist.ReduceOp.MAX)
    st = layer.local_stage_ms or [0.0] * 5
    rows, active = layer.last_local_rows, layer.last_local_active
    tile_n = fmoe_b200.tile_n(fmoe_b200.make_problem(layer.last_local_tokens, 256, per, H, I))
    g1, g2 = kernel_rooflines(rows, active, st, hbm, fp8, fp8_src, hbm_src, tile_n)
    g1["stage_us"] = dict(zip(fmoe_b200.StageTimer.STAGES, [round(x * 1e3, 1) for x in st]))
    g1["gemm2"] = g2
    g1["traffic"] = None
    g1["rank"] = rank
    parity = ep_parity(out, acts, weights, world, rank, per, layer)
    e2e_ms, e2e_serial, h2d, d2h = time_e2e(acts, weights, args.steps, args.warmup,
                                            lambda *a, out=None: layer.forward(*a))
    line = base_line(args, world, T, ms_per_step,
                     layer_config(T, world, args.exchange, args.placement, args.ep_host_sync))
    line.update({
        "breakdown_ms_max_over_ranks": {"route": round(float(br[0]), 3),
                                        "dispatch": round(float(br[1]), 3),
                                        "compute": round(float(br[2]), 3),
                                        "combine": round(float(br[3]), 3)},
        "roofline": g1, "clocks": clk.summary(), "ep_parity": parity,
        "e2e": {"value": round(world * T / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "mode": "per rank: copies on separate H2D / D2H streams, overlapping the "
                        "neighbouring steps (2 buffer slots)",
                "serial_value": round(world * T / (e2e_serial * 1e-3), 1)},
        # routing, send plan, pack, unpack, the operator's 5 kernels, (P2P: return), combine
        "gpu_launches": (10 + (args.exchange == "p2p")) * args.steps,
    })
    layer.close()
    return line


def base_line(args, world, T, ms_per_step, config):
    return {
        "metric": "MoE layer tokens/s (DS-V3 full 256-expert layer, 4096 tokens per GPU)",
        "value": round(world * T / (ms_per_step * 1e-3), 1), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4), "us_per_call": round(ms_per_step * 1e3, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3 x e4m3 -> fp32 (tcgen05 kind::f8f6f4), fp32 block-scale promotion",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights, FP8 128-block scales)",
        "config": config,
    }


SWEEP_CASES = [("config1", 1, 0), ("config1", 4, 0), ("config1", 16, 0), ("config1", 64, 0),
               ("config2", 512, 0), ("config2", 2048, 0), ("config2", 4096, 0),
               ("config2", 8192, 0), ("config4", 4096, 8)]


def sweep_cases(args):
    if args.sweep_tokens:
        return [("config1" if T <= 64 else "config2", T, 0)
                for T in (int(x) for x in args.sweep_tokens.split(",") if x)]
    return SWEEP_CASES


def sweep_ours(args, w32, peaks, flush):
    """Configs 1, 2 and 4 on one 32-expert slice (local_expert_offset 0). `--sweep-tiles`
    lists the token tiles timed per case (0 = the autotune table); tiles above 16 are
    skipped below T = 64, and 128 below T = 512."""
    hbm, fp8, hbm_src, fp8_src = peaks
    wargs = [w32[k] for k in W.OPERATOR_ARGS[4:]]
    # the same weights pre-laid-out (fmoe_prelayout_weights): each case is also timed on them
    w13p, w2p = fmoe_b200.prelayout_weights(w32["gemm1_weights"], w32["gemm2_weights"])
    pargs = [w13p, w32["gemm1_weights_scale"], w2p, w32["gemm2_weights_scale"]]
    tiles = tuple(int(x) for x in args.sweep_tiles.split(","))
    res = []
    for cfg, T, skew in sweep_cases(args):
        acts = W.make_activations(W.DSV3, T, args.seed, device="cuda", skew_hot=skew)
        rows, active = routed_stats(acts, 0, 32)
        a4 = [acts[k] for k in W.OPERATOR_ARGS[:4]]
        out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        for tile in tiles:
            if (tile > 16 and T < 64) or (tile == 128 and T < 512):
                continue
            fn = lambda: fmoe_b200.kernel(*a4, *wargs, 0, RSF, out=out, tile_n=tile)  # noqa
            stage_ms, eager = time_stages(fn, 10, flush)
            ms = time_graph(fn, 10, 3, flush)
            t = statistics.median(ms)
            fnp = lambda: fmoe_b200.kernel(*a4, *pargs, 0, RSF, out=out, tile_n=tile,  # noqa
                                           prelaid=True)
            t_pre = statistics.median(time_graph(fnp, 10, 3, flush))
            tn = tile or fmoe_b200.tile_n(fmoe_b200.make_problem(T, 256, 32, H, I))
            g1, g2 = kernel_rooflines(rows, active, stage_ms, hbm, fp8, fp8_src, hbm_src, tn)
            lay = roofline("whole layer", layer_bytes(T, active), rows * FLOP_PER_ROW, t, hbm,
                           fp8, fp8_src, hbm_src)
            res.append({"config": cfg, "T": T, "skew_hot": skew, "rows": rows,
                        "active_experts": active, "tile_n": tn,
                        "us_per_call": round(t * 1e3, 1),
                        "us_per_call_prelaid_weights": round(t_pre * 1e3, 1),
                        "us_per_call_eager": round(statistics.median(eager) * 1e3, 1),
                        "tokens_per_s": round(T / (t * 1e-3), 1),
                        "roofline": {k: lay[k] for k in ("bound", "achieved", "peak", "unit",
                                                          "frac")},
                        "hbm_frac": lay["hbm_frac"], "fp8_frac": lay["fp8_frac"],
                        "gemm1": {k: g1[k] for k in ("bound", "frac", "us", "hbm_frac",
                                                     "fp8_frac")},
                        "gemm2": {k: g2[k] for k in ("bound", "frac", "us", "hbm_frac",
                                                     "fp8_frac")},
                        "stage_us": dict(zip(fmoe_b200.StageTimer.STAGES,
                                             [round(x * 1e3, 1) for x in stage_ms]))})
        del acts
        torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------------------------- reference arm
def reference_kernel():
    so = ROOT / "oracle" / "_ref" / "ref_kernel.so"
    if not so.exists():
        return None, "reference kernel not built (oracle/build_ref.sh needs the source)"
    import tvm_ffi

    return tvm_ffi.load_module(str(so))["kernel"], None


def run_reference(args, world, rank, local, flush):
    """The reference operator on the same layer workload: eight 32-expert slice calls per
    step on every rank (each rank holds all 256 experts), slices summed by the caller."""
    kern, why = reference_kernel()
    head = {"metric": "MoE layer tokens/s (DS-V3 full 256-expert layer, 4096 tokens per GPU)",
            "impl": "reference"}
    if kern is None:
        return dict(head, unavailable=why)
    T = args.tokens or LAYER_TOKENS
    weights = layer_weights(args.seed, 0, 256)
    acts = layer_activations(args.seed, rank, T)
    a4 = [acts[k] for k in W.OPERATOR_ARGS[:4]]
    sl = [[weights[k][32 * s:32 * s + 32] for k in W.OPERATOR_ARGS[4:]] for s in range(8)]
    acc = torch.empty(T, H, dtype=torch.float32, device="cuda")

    def step():
        acc.zero_()
        for s in range(8):
            o = torch.from_dlpack(kern(*a4, *sl[s], 32 * s, RSF))
            acc.add_(o.float())
        return acc.to(torch.bfloat16)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    pairs = []
    with ClockSampler(gpu_index_of(local)) as clk:
        for _ in range(args.steps):
            flush_l2(flush)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            step()
            e1.record()
            pairs.append((e0, e1))
        torch.cuda.synchronize()
    ms_per_step = max_over_ranks(sum(x.elapsed_time(y) for x, y in pairs)) / args.steps
    line = dict(head)
    line.update(base_line(args, world, T, ms_per_step, layer_config(T, world, args.exchange)))
    line["impl"] = "reference"
    line["config"]["parallelism"] = (f"replicas x{world} (the reference has no expert "
                                     "parallelism: every rank holds all 256 experts)"
                                     if world > 1 else line["config"]["parallelism"])
    for k in ("collectives", "placement"):  # no exchange between the reference's replicas
        line["config"].pop(k, None)
    line.update({
        "dtype": "e4m3 x e4m3 -> fp32 (reference: fp32 SIMT / f16 and tf32-class mma.sync)",
        "runs_on": ("cuda (B200): the reference implements the path only in CUDA "
                    "(solution/cuda/kernel.cu); eight local_expert_offset slice calls per step, "
                    "each ending in its own stream synchronisation, slices summed in fp32"),
        "clocks": clk.summary(),
        "e2e": {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    })
    del acts
    if world == 1 and not args.no_sweep:
        w32 = [weights[k][:32] for k in W.OPERATOR_ARGS[4:]]
        line["sweep"] = sweep_reference(args, kern, w32, flush)
    return line


def sweep_reference(args, kern, w32, flush):
    """The reference operator on the sweep's cases (one 32-expert slice, offset 0)."""
    res = []
    for cfg, T, skew in sweep_cases(args):
        acts = W.make_activations(W.DSV3, T, args.seed, device="cuda", skew_hot=skew)
        a4 = [acts[k] for k in W.OPERATOR_ARGS[:4]]
        for _ in range(3):
            kern(*a4, *w32, 0, RSF)
        torch.cuda.synchronize()
        ms = []
        for _ in range(10):
            flush_l2(flush)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            kern(*a4, *w32, 0, RSF)
            e1.record()
            torch.cuda.synchronize()
            ms.append(e0.elapsed_time(e1))
        t = statistics.median(ms)
        res.append({"config": cfg, "T": T, "skew_hot": skew, "ref_us_per_call": round(t * 1e3, 1),
                    "tokens_per_s": round(T / (t * 1e-3), 1)})
        del acts
        torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------------------------- one slice
def run_slice(args, peaks, flush):
    """`--workload slice`: one 32-expert slice at --tokens / --skew (configs 1, 2, 4)."""
    hbm, fp8, hbm_src, fp8_src = peaks
    T = args.tokens or 64
    w32 = layer_weights(args.seed, 0, 32)
    acts = W.make_activations(W.DSV3, T, args.seed, device="cuda", skew_hot=args.skew)
    rows, active = routed_stats(acts, 0, 32)
    a4 = [acts[k] for k in W.OPERATOR_ARGS[:4]]
    wargs = [w32[k] for k in W.OPERATOR_ARGS[4:]]
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    fn = lambda: fmoe_b200.kernel(*a4, *wargs, 0, RSF, out=out)  # noqa: E731
    fn()
    torch.cuda.synchronize()
    stage_ms, eager = time_stages(fn, args.steps, flush)
    with ClockSampler(gpu_index_of(0)) as clk:
        ms = time_graph(fn, args.steps, args.warmup, flush)
    t = sum(ms) / len(ms)
    tn = fmoe_b200.tile_n(fmoe_b200.make_problem(T, 256, 32, H, I))
    g1, g2 = kernel_rooflines(rows, active, stage_ms, hbm, fp8, fp8_src, hbm_src, tn)
    g1["gemm2"] = g2
    g1["traffic"] = stored_traffic(f"gemm1_T{T}" + (f"_hot{args.skew}" if args.skew else ""))
    cfg = {"workload": (f"config4_dsv3_T{T}_hot{args.skew}" if args.skew else
                        f"config{1 if T <= 64 else 2}_dsv3_slice_T{T}"),
           "tokens_per_rank": T, "hidden": H, "intermediate": I, "experts": 256,
           "local_experts": 32, "routed_rows": rows, "active_experts": active, "tile_n": tn}
    line = base_line(args, 1, T, t, cfg)
    line["metric"] = "MoE layer tokens/s (DS-V3, one 32-expert slice)"
    line.update({"roofline": g1, "clocks": clk.summary(),
                 "us_per_call_eager": round(statistics.median(eager) * 1e3, 1),
                 "stage_us": dict(zip(fmoe_b200.StageTimer.STAGES,
                                      [round(x * 1e3, 1) for x in stage_ms])),
                 "gpu_launches": 5 * args.steps})
    return line


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
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("layer", "slice"), default="layer",
                    help="layer: config 3, the full 256-expert layer (the headline); "
                         "slice: one 32-expert slice at --tokens / --skew")
    ap.add_argument("--tokens", type=int, default=None,
                    help="tokens per rank (layer: 4096; slice: 64)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--skew", type=int, default=0,
                    help="slice workload: route every token onto this many hot local experts "
                         "(config 4: 8); 0 = grouped top-k over random logits")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--placement", choices=("local", "balanced", "contiguous"),
                    default="local", help="N>1: expert placement over the ranks")
    ap.add_argument("--placement-search", choices=("max-rank", "pairs"), default="max-rank",
                    help="N>1, --placement local: swap search of the locality placement")
    ap.add_argument("--ep-separate-return", action="store_true",
                    help="N>1: return the partial rows with a separate kernel after the "
                         "operator instead of from the operator's combine")
    ap.add_argument("--ep-host-sync", action="store_true",
                    help="N>1: size each step's exchange on the host (one device-to-host read "
                         "of the counts per step) instead of the sync-free device offsets")
    ap.add_argument("--exchange", choices=("p2p", "nccl"), default="p2p",
                    help="expert-parallel runs (N > 1): rows over peer memory or NCCL all-to-all")
    ap.add_argument("--sweep-tiles", default="0",
                    help="comma-separated token tiles timed per sweep case (0 = autotune)")
    ap.add_argument("--sweep-tokens", default="",
                    help="comma-separated token counts replacing the sweep's cases")
    args = ap.parse_args()
    assert args.warmup >= 3, "at least 3 warm-up steps"

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=120))
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    try:
        if args.impl == "reference":
            line = run_reference(args, world, rank, local, flush)
        else:
            hbm, bf16, hbm_src = load_peaks()
            fp8 = measure_fp8_peak()
            fp8 = max_over_ranks(fp8) if world > 1 else fp8
            peaks = (hbm, fp8, f"{hbm_src} (MEASURED_PEAKS.json hbm_gbs)",
                     "measured live (fmoe_probe_fp8_mma_rate: tcgen05 M128N256K32 "
                     "kind::f8f6f4, one CTA per SM)")
            if world > 1:
                line = run_ep(args, world, rank, local, peaks)
            elif args.workload == "slice":
                line = run_slice(args, peaks, flush)
            else:
                line = run_layer_single(args, peaks, flush)
            line["peaks"] = {"hbm_gbs": hbm, "fp8_dense_tflops_measured": round(fp8, 1),
                             "bf16_tflops": bf16, "bf16_source": hbm_src}
        if rank == 0:
            emit(line)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
