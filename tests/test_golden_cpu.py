"""The CPU oracle against golden outputs of the reference operator itself.

The fixtures in tests/golden/ were produced by running the reference
`solution/cuda/kernel.cu` on a B200 (tests/golden/make_ref_goldens.py); the inputs are
regenerated here from their seeds. The tie-heavy case pins the lowest-index tie rule of
the reference's routing (kernel.cu:444-495) end to end.
"""
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).parent / "golden"
sys.path.insert(0, str(GOLDEN))

FIXTURES = sorted(GOLDEN.glob("*.npz"))


@pytest.mark.parametrize("path", FIXTURES, ids=[p.stem for p in FIXTURES])
def test_oracle_matches_reference_golden(oracle_mod, path):
    from make_ref_goldens import case_inputs
    from fmoe_b200 import workloads as W

    d = np.load(path)
    T, seed, ties = int(d["tokens"]), int(d["seed"]), bool(d["ties"])
    inp, experts = case_inputs(T, seed, ties)
    assert experts == [int(e) for e in d["experts"]], "routing chose different experts"
    geo = W.DSV3
    out = oracle_mod.moe_forward(*W.operator_args(inp), int(d["local_expert_offset"]),
                                 float(d["routed_scaling_factor"]), geo.n_group,
                                 geo.topk_group, geo.top_k)
    ref = torch.from_numpy(d["out_bf16_bits"]).view(torch.bfloat16).float()
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)
    rel = (out.float() - ref).norm() / ref.norm().clamp_min(1e-12)
    assert rel < 1e-2


def test_fixtures_present():
    assert len(FIXTURES) >= 3, "run tests/golden/make_ref_goldens.py on a B200"
