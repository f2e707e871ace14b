"""fmoe_route_static(): routing with no workspace argument and no allocation.

This entry point is for callers that cannot give the library scratch memory: plugin
interfaces that pass only the call's tensors, and engines that reserve all device memory
at start-up and forbid allocation afterwards. Its scratch is a fixed device array inside
the library. This test calls it through the C ABI twice in a row, on different inputs, and
checks every result against the workspace-based fmoe_route(). Routing is integer/index
work plus IEEE single-precision arithmetic, so the comparison is bit for bit.

Kept in its own file, named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(T, E, seed):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(T, E, generator=g).cuda()
    bias = (torch.randn(E, generator=g) * 0.1).to(torch.bfloat16).cuda()
    return logits, bias


def _route_static(fmoe, prob, logits, bias, idx, w):
    lib = fmoe.load_library()
    lib.fmoe_route_static.argtypes = [ctypes.POINTER(fmoe.FmoeProblem), ctypes.c_void_p,
                                      ctypes.c_void_p, ctypes.POINTER(fmoe.FmoeRouteOut),
                                      ctypes.c_void_p]
    out = fmoe.FmoeRouteOut(idx.data_ptr(), w.data_ptr())
    stream = torch.cuda.current_stream().cuda_stream
    return lib.fmoe_route_static(ctypes.byref(prob), logits.data_ptr(), bias.data_ptr(),
                                 ctypes.byref(out), stream)


# (E_global, E_local, first call's tokens, second call's tokens). The largest case fills the
# whole static scratch (8192 tokens: 512 CTAs x 64 experts of per-CTA counts and bases) and
# is followed by a small one, so stale entries from the large call would show up.
@pytest.mark.parametrize("E,E_local,T1,T2", [(256, 32, 64, 4096), (16, 16, 7, 100),
                                             (256, 64, 8192, 64), (256, 64, 8192, 8192)])
def test_route_static_matches_route_twice(fmoe, E, E_local, T1, T2):
    for call, T in enumerate((T1, T2)):
        logits, bias = _inputs(T, E, seed=40 + call)
        prob = fmoe.make_problem(T, E, E_local, 7168 if E == 256 else 256,
                                 2048 if E == 256 else 128)
        idx = torch.full((T, prob.top_k), -7, dtype=torch.int32, device="cuda")
        w = torch.full((T, prob.top_k), -7.0, dtype=torch.float32, device="cuda")
        rc = _route_static(fmoe, prob, logits, bias, idx, w)
        assert rc == fmoe.FMOE_OK, fmoe.load_library().fmoe_last_error()
        ref_idx, ref_w = fmoe.route(logits, bias, prob.n_group, prob.topk_group, prob.top_k,
                                    prob.routed_scaling_factor, num_local_experts=E_local,
                                    local_expert_offset=prob.local_expert_offset)
        torch.cuda.synchronize()
        assert torch.equal(idx, ref_idx)
        assert np.array_equal(w.cpu().numpy().view(np.uint32),
                              ref_w.cpu().numpy().view(np.uint32))


def test_route_static_rejects_oversized(fmoe):
    T = 8193
    logits, bias = _inputs(T, 256, seed=1)
    prob = fmoe.make_problem(T, 256, 32, 7168, 2048)
    idx = torch.empty(T, 8, dtype=torch.int32, device="cuda")
    w = torch.empty(T, 8, dtype=torch.float32, device="cuda")
    rc = _route_static(fmoe, prob, logits, bias, idx, w)
    assert rc == fmoe.FMOE_ERR_VALUE
    assert b"exceeds the static scratch limit" in fmoe.load_library().fmoe_last_error()


def test_route_static_rejects_too_many_local_experts(fmoe):
    T = 64
    logits, bias = _inputs(T, 256, seed=2)
    prob = fmoe.make_problem(T, 256, 65, 7168, 2048)
    idx = torch.empty(T, 8, dtype=torch.int32, device="cuda")
    w = torch.empty(T, 8, dtype=torch.float32, device="cuda")
    rc = _route_static(fmoe, prob, logits, bias, idx, w)
    assert rc == fmoe.FMOE_ERR_VALUE
    assert b"beyond the static limits" in fmoe.load_library().fmoe_last_error()
