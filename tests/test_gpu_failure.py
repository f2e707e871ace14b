"""Failure detection on the GPU without a fault: the bounded waits of the GEMM kernels are
made to run out (an mbarrier nobody arrives on, a global flag nobody sets) with a short
limit; the kernel must report both expiries and return, and the context must stay usable
for the operator right after. No test here faults, traps or hangs a GPU."""
import pytest
import torch

from fmoe_b200 import workloads as W

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("timeout_ns", [2_000_000, 10_000_000])
def test_bounded_waits_expire_and_report(fmoe, timeout_ns):
    r = fmoe.selftest_wait_timeout(timeout_ns)
    assert r["expired_mask"] == 3
    for k in ("mbarrier_wait_ns", "flag_wait_ns"):
        assert timeout_ns <= r[k] < timeout_ns + 50_000_000, r


def test_context_usable_after_expired_waits(fmoe, oracle_mod):
    fmoe.selftest_wait_timeout(2_000_000)
    geo = W.TINY
    inp = W.make_inputs(geo, 16, seed=5)
    gpu = {k: v.cuda() for k, v in inp.items() if isinstance(v, torch.Tensor)}
    out = fmoe.kernel(*W.operator_args(gpu), 0, 2.5)
    torch.cuda.synchronize()
    ref = oracle_mod.moe_forward(*W.operator_args(inp), 0, 2.5, geo.n_group, geo.topk_group,
                                 geo.top_k)
    torch.testing.assert_close(out.float().cpu(), ref.float(), atol=2e-2, rtol=2e-2)
    prob = fmoe.make_problem(16, geo.num_experts, geo.num_local, geo.hidden, geo.inter)
    ws = fmoe.Workspace.get(torch.device("cuda", torch.cuda.current_device()),
                            fmoe.workspace_bytes(prob))
    assert fmoe.read_device_error(prob, ws) == 0


def test_selftest_rejects_bad_limits(fmoe):
    with pytest.raises(ValueError):
        fmoe.selftest_wait_timeout(0)
    with pytest.raises(ValueError):
        fmoe.selftest_wait_timeout(10**9)
