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


# ---- device errors reach the caller (fmoe_poll_device_error), without a fault -------------
# The error is planted on the host (fmoe_selftest_inject_device_error): the next call's
# routing kernel ORs the bits into the call's device error word, as an expired wait would,
# and the call's last kernel passes the word on to the host. Nothing waits or faults.
_ERR_TIMEOUT_MMA = 1 << 1


def _tiny_gpu(seed=3):
    geo = W.TINY
    inp = W.make_inputs(geo, 16, seed=seed)
    return inp, {k: v.cuda() for k, v in inp.items() if isinstance(v, torch.Tensor)}


def test_device_error_raises_at_the_next_call(fmoe, oracle_mod):
    geo = W.TINY
    inp, gpu = _tiny_gpu()
    assert fmoe.poll_device_error() == 0
    fmoe.inject_device_error(_ERR_TIMEOUT_MMA)
    out = fmoe.kernel(*W.operator_args(gpu), 0, 2.5)  # returns: the call is asynchronous
    torch.cuda.synchronize()
    ref = oracle_mod.moe_forward(*W.operator_args(inp), 0, 2.5, geo.n_group, geo.topk_group,
                                 geo.top_k)
    torch.testing.assert_close(out.float().cpu(), ref.float(), atol=2e-2, rtol=2e-2)
    with pytest.raises(RuntimeError, match="device error 0x2"):
        fmoe.kernel(*W.operator_args(gpu), 0, 2.5)
    # reported once: the call after that runs normally
    out2 = fmoe.kernel(*W.operator_args(gpu), 0, 2.5)
    torch.cuda.synchronize()
    assert torch.equal(out2, out)
    assert fmoe.poll_device_error() == 0


def test_device_error_check_raises_for_the_same_call(fmoe):
    _, gpu = _tiny_gpu(4)
    fmoe.kernel(*W.operator_args(gpu), 0, 2.5, check=True)  # clean call: no error
    fmoe.inject_device_error(_ERR_TIMEOUT_MMA)
    with pytest.raises(fmoe.DeviceError, match="this call"):
        fmoe.kernel(*W.operator_args(gpu), 0, 2.5, check=True)
    assert fmoe.poll_device_error() == 0


def test_device_error_forward_routed_and_graph_cache(fmoe):
    # repeated identical calls replay from the library's graph cache; an injected error
    # forces that one call to run eagerly and is still reported
    _, gpu = _tiny_gpu(5)
    args = W.operator_args(gpu)
    for _ in range(3):
        fmoe.kernel(*args, 0, 2.5)
    torch.cuda.synchronize()
    fmoe.inject_device_error(_ERR_TIMEOUT_MMA | 1)
    fmoe.kernel(*args, 0, 2.5)
    torch.cuda.synchronize()
    assert fmoe.poll_device_error() == 3
    geo = W.TINY
    idx, w = fmoe.route(gpu["routing_logits"], gpu["routing_bias"], geo.n_group,
                        geo.topk_group, geo.top_k, 2.5, num_local_experts=geo.num_local)
    fmoe.inject_device_error(_ERR_TIMEOUT_MMA)
    fmoe.forward_routed(idx, w, gpu["hidden_states"], gpu["hidden_states_scale"], *args[4:], 0,
                        geo.num_experts, n_group=geo.n_group, topk_group=geo.topk_group)
    with pytest.raises(RuntimeError, match="device error"):
        fmoe.forward_routed(idx, w, gpu["hidden_states"], gpu["hidden_states_scale"], *args[4:],
                            0, geo.num_experts, n_group=geo.n_group, topk_group=geo.topk_group)
    assert fmoe.poll_device_error() == 0


def test_device_error_tvm_ffi_binding_raises(fmoe):
    pytest.importorskip("tvm_ffi")
    if not fmoe.TVM_FFI_LIB_PATH.exists():
        pytest.skip("TVM-FFI binding not built")
    kern = fmoe.load_tvm_ffi_kernel()
    _, gpu = _tiny_gpu(6)
    args = W.operator_args(gpu)
    kern(*args, 0, 2.5)
    torch.cuda.synchronize()
    fmoe.inject_device_error(_ERR_TIMEOUT_MMA)
    kern(*args, 0, 2.5)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="device error 0x2"):
        kern(*args, 0, 2.5)
    kern(*args, 0, 2.5)
    torch.cuda.synchronize()
    assert fmoe.poll_device_error() == 0


def test_fp8_mma_rate_probe(fmoe):
    r = fmoe.probe_fp8_mma_rate(16384)
    # dense FP8 on a B200: 4.5 PF/s nominal at the boost clock; a throttled GPU runs lower
    assert 1000.0 < r["tflops"] < 5200.0, r
    assert r["ms"] > 0.0
    with pytest.raises(ValueError):
        fmoe.probe_fp8_mma_rate(1)
