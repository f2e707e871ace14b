"""Generate golden fixtures from the reference operator itself.

Runs the reference YuWei-CH/Fused-MoE-YWS `solution/cuda/kernel.cu` (compiled in place
by `oracle/build_ref.sh` into `oracle/_ref/ref_kernel.so`) on a B200 and stores its bf16
outputs as small `.npz` fixtures next to this script. Inputs are not stored: they are
regenerated on the CPU from the recorded seed by `fmoe_b200.workloads` (torch CPU
generators are deterministic), and only the local experts the oracle routes to receive
weights; the other experts are zero and unread.

Usage (on a GPU box, from the repository root):
    python tests/golden/make_ref_goldens.py [--out-dir DIR]

`tests/test_golden_cpu.py` checks the CPU oracle against these fixtures.
"""
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "fused-moe-yws_b200"))
sys.path.insert(0, str(ROOT))

from fmoe_b200 import workloads as W  # noqa: E402

# (name, tokens, seed, tie_heavy): tie_heavy logits are multiples of 0.5 with zero bias, so
# group scores and expert scores tie and the reference's lowest-index rule decides.
CASES = [("dsv3_T4_s101", 4, 101, False), ("dsv3_T16_s102", 16, 102, False),
         ("dsv3_T16_s103_ties", 16, 103, True)]


def case_inputs(T, seed, ties, device="cpu"):
    import oracle

    geo = W.DSV3
    acts = W.make_activations(geo, T, seed, device="cpu")
    if ties:
        acts["routing_logits"] = torch.round(acts["routing_logits"] * 2.0) / 2.0
        acts["routing_bias"] = torch.zeros_like(acts["routing_bias"])
    idx, _ = oracle.route(acts["routing_logits"], acts["routing_bias"], geo.n_group,
                          geo.topk_group, geo.top_k, 2.5)
    experts = sorted({int(e) for e in idx.ravel() if 0 <= e < geo.num_local})
    acts.update(W.make_weights(geo, seed, device="cpu", experts=experts))
    if device != "cpu":
        acts = {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in acts.items()}
    return acts, experts


def main():
    import argparse

    import tvm_ffi

    ap = argparse.ArgumentParser()
    ap.add_argument("--out-dir", default=str(Path(__file__).parent))
    out_dir = Path(ap.parse_args().out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)

    so = ROOT / "oracle" / "_ref" / "ref_kernel.so"
    kern = tvm_ffi.load_module(str(so))["kernel"]
    for name, T, seed, ties in CASES:
        inp, experts = case_inputs(T, seed, ties, device="cuda")
        out = torch.from_dlpack(kern(*W.operator_args(inp), 0, 2.5))
        torch.cuda.synchronize()
        np.savez_compressed(out_dir / f"{name}.npz",
                            out_bf16_bits=out.cpu().view(torch.int16).numpy(),
                            tokens=T, seed=seed, ties=ties, experts=np.array(experts),
                            local_expert_offset=0, routed_scaling_factor=2.5)
        print(name, "experts", experts, "mean|out|", float(out.float().abs().mean()))


if __name__ == "__main__":
    main()
