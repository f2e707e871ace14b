"""bench.py without a GPU: its command line, the algorithmic byte and FLOP constants behind
the roofline, and the skewed workload (config 4) it times."""
import subprocess
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent


def test_help_lists_the_contract_options():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"], capture_output=True,
                       text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr
    # stdout is kept for the one JSON line, so everything else (help included) goes to stderr
    text = r.stdout + r.stderr
    for opt in ("--gpus", "--steps", "--warmup", "--impl", "--tokens", "--skew", "--exchange",
                "--sweep-tiles", "--sweep-tokens", "--no-sweep", "--no-cpu", "--placement",
                "--placement-search", "--ep-host-sync", "--ep-separate-return"):
        assert opt in text, opt


def test_layer_config_names_the_workload_and_the_exchange():
    import bench

    one = bench.layer_config(4096, 1, "p2p")
    assert one["workload"] == "config3_dsv3_full_layer" and one["experts_per_rank"] == 256
    assert "collectives" not in one and "placement" not in one  # no exchange on one GPU
    eight = bench.layer_config(4096, 8, "p2p")
    assert eight["experts_per_rank"] == 32 and eight["parallelism"] == "ep8"
    assert eight["placement"].startswith("local") and "no host round" in eight["collectives"]
    assert bench.layer_config(4096, 8, "p2p", "contiguous")["placement"].startswith("contiguous")
    assert "host each step" in bench.layer_config(4096, 2, "p2p", "local", True)["collectives"]
    assert "all-to-all" in bench.layer_config(4096, 2, "nccl")["collectives"]


def test_roofline_constants_match_the_dsv3_shapes():
    import bench

    H, I, E_local = 7168, 2048, 32
    w13, w2 = 2 * I * H, H * I                                   # FP8 bytes per expert
    s13, s2 = (2 * I // 128) * (H // 128) * 4, (H // 128) * (I // 128) * 4
    assert bench.FLOP_PER_ROW == 2 * H * 2 * I + 2 * I * H
    assert bench.GEMM1_FLOP_PER_ROW == 2 * H * 2 * I
    assert bench.BYTES_PER_EXPERT == w13 + w2 + s13 + s2
    assert bench.GEMM1_BYTES_PER_EXPERT == w13 + s13
    # GEMM1 per routed row: the FP8 row and its scales in, the hi/lo intermediate and its
    # scales out
    assert bench.GEMM1_BYTES_PER_ROW == H + (H // 128) * 4 + 2 * I + (I // 128) * 4
    assert E_local * bench.BYTES_PER_EXPERT == 1_409_630_208  # the whole 32-expert slice
    assert bench.L2_FLUSH_BYTES > 126 * 2**20                  # larger than the B200's L2


def test_skewed_workload_routes_every_token_to_its_hot_experts(oracle_mod):
    from fmoe_b200 import workloads as W

    geo = W.DSV3
    for hot_n in (8, 32):
        acts = W.make_activations(geo, 48, seed=5, device="cpu", skew_hot=hot_n)
        hot = set(acts["hot_experts"])
        assert len(hot) == hot_n and all(0 <= e < geo.num_local for e in hot)
        idx, _ = oracle_mod.route(acts["routing_logits"], acts["routing_bias"], geo.n_group,
                                  geo.topk_group, geo.top_k, 2.5)
        local = idx[(idx >= 0) & (idx < geo.num_local)]
        # every selection lands on a hot expert: all top_k when there are at least top_k
        assert set(np.unique(local).tolist()) <= hot
        assert local.size == 48 * geo.top_k
