"""CPU checks of the oracle: hand-made routing known-answer tests, the exact sigmoid,
the stable row plan and the dequantise-to-fp32 restatement of the operator.

The routing KATs below are derived by hand from the reference algorithm
(solution/cuda/kernel.cu:408-516): group score = sum of the two largest biased scores,
ties keep the lower group / expert index (strict '>' comparisons at kernel.cu:451, :478),
weights come from the unbiased sigmoid scores.
"""
import math

import numpy as np
import pytest
import torch

from fmoe_b200 import workloads as W


def bf16(vals):
    return torch.tensor(vals, dtype=torch.float32).to(torch.bfloat16)


# (name, E, n_group, topk_group, top_k, logits row, bias row, expected idx, expected w)
def _kats():
    kats = []
    # 1. everything equal: lowest groups, lowest experts; w = 0.5 / (K * 0.5) * 2.5
    kats.append(("all_equal_tiny", 16, 4, 2, 4, [0.0] * 16, [0.0] * 16, [0, 1, 2, 3],
                 [0.625] * 4))
    kats.append(("all_equal_dsv3", 256, 8, 4, 8, [0.0] * 256, [0.0] * 256, list(range(8)),
                 [0.3125] * 8))
    # 2. the bias decides the selection, the weights stay on the unbiased scores
    b = [0.0] * 256
    for e in range(200, 208):
        b[e] = 1.0
    kats.append(("bias_selects_dsv3", 256, 8, 4, 8, [0.0] * 256, b, list(range(200, 208)),
                 [0.3125] * 8))
    # 3. group score is the top-2 SUM: group 1 (1.1 + 1.1) beats group 0 (1.5 + 0.5)
    b = [0.0] * 16
    b[0], b[4], b[5], b[8], b[9] = 1.0, 0.6, 0.6, 0.3, 0.3
    kats.append(("top2_sum_tiny", 16, 4, 2, 4, [0.0] * 16, b, [0, 4, 5, 1], [0.625] * 4))
    # 4. a -inf bias removes a group; the remaining ties keep the lower groups
    b = [0.0] * 16
    for e in range(4):
        b[e] = -math.inf
    kats.append(("neg_inf_group_tiny", 16, 4, 2, 4, [0.0] * 16, b, [4, 5, 6, 7], [0.625] * 4))
    # 5. only two finite candidates: remaining slots stay -1 with weight 0
    b = [-math.inf] * 16
    b[4] = b[5] = 0.0
    w = 0.5 / (1.0 + 1e-20) * 2.5
    kats.append(("too_few_candidates_tiny", 16, 4, 2, 4, [0.0] * 16, b, [4, 5, -1, -1],
                 [w, w, 0.0, 0.0]))
    # 6. a NaN logit is never selected
    lg = [0.0] * 16
    lg[0] = math.nan
    kats.append(("nan_logit_tiny", 16, 4, 2, 4, lg, [0.0] * 16, [1, 2, 3, 4], [0.625] * 4))
    # 7. logit order decides inside kept groups; larger logit first
    lg = [0.0] * 16
    lg[6], lg[2], lg[3] = 3.0, 2.0, 2.0
    s6 = 1.0 / (1.0 + math.exp(-3.0))
    s2 = 1.0 / (1.0 + math.exp(-2.0))
    tot = np.float32(np.float32(np.float32(s6) + np.float32(s2)) + np.float32(s2)) + np.float32(0.5)
    kats.append(("logit_order_tiny", 16, 4, 2, 4, lg, [0.0] * 16, [6, 2, 3, 0],
                 [float(np.float32(s6) / tot * np.float32(2.5)),
                  float(np.float32(s2) / tot * np.float32(2.5)),
                  float(np.float32(s2) / tot * np.float32(2.5)),
                  float(np.float32(0.5) / tot * np.float32(2.5))]))
    return kats


@pytest.mark.parametrize("kat", _kats(), ids=lambda k: k[0])
def test_routing_kat(oracle_mod, kat):
    name, E, ng, kg, k, lg, b, exp_idx, exp_w = kat
    logits = torch.tensor([lg], dtype=torch.float32)
    idx, w = oracle_mod.route(logits, bf16(b), ng, kg, k, 2.5)
    assert idx[0].tolist() == exp_idx
    # exact where the expected value is a dyadic rational, 1e-6 relative otherwise
    np.testing.assert_allclose(w[0], np.array(exp_w, np.float32), rtol=1e-6, atol=0)


def test_sigmoid_accuracy(oracle_mod):
    x = np.linspace(-80, 80, 40001, dtype=np.float32)
    s = oracle_mod.sigmoid(x)
    ref = 1.0 / (1.0 + np.exp(-x.astype(np.float64)))
    assert np.max(np.abs(s - ref) / ref) < 4 * 2.0 ** -24
    assert oracle_mod.sigmoid(np.array([0.0], np.float32))[0] == 0.5
    assert oracle_mod.sigmoid(np.array([200.0], np.float32))[0] == 1.0
    assert oracle_mod.sigmoid(np.array([-200.0], np.float32))[0] == 0.0


@pytest.mark.parametrize("geo", [W.TINY, W.DSV3], ids=["tiny", "dsv3"])
def test_route_matches_definition_style(oracle_mod, geo):
    """Exact-sigmoid routing agrees with a torch.sigmoid/topk definition on random data
    (selection sets may only differ on near ties; none occur at these sizes)."""
    acts = W.make_activations(geo, 512, seed=3)
    ng, kg, k = geo.n_group, geo.topk_group, geo.top_k
    idx, w = oracle_mod.route(acts["routing_logits"], acts["routing_bias"], ng, kg, k, 2.5)
    idx2, w2 = oracle_mod.route_definition(acts["routing_logits"], acts["routing_bias"], ng, kg,
                                           k, 2.5)
    assert (np.sort(idx, 1) == np.sort(idx2, 1)).all()
    order = np.argsort(idx, 1)
    order2 = np.argsort(idx2, 1)
    np.testing.assert_allclose(np.take_along_axis(w, order, 1),
                               np.take_along_axis(w2, order2, 1), rtol=2e-6)


def test_plan_stable_order(oracle_mod):
    rng = np.random.default_rng(0)
    T, K, EL = 50, 8, 32
    idx = rng.integers(0, 64, size=(T, K)).astype(np.int32)
    p = oracle_mod.plan(idx, EL, 16, row_cap=T * K + 16 * EL)
    cnt = p["expert_cnt"]
    off = p["expert_off"]
    for le in range(EL):
        rows = p["row_token"][off[le]:off[le] + cnt[le]]
        toks = [t for t in range(T) for k in range(K) if idx[t, k] == le + 16]
        assert rows.tolist() == toks
        assert (p["row_token"][off[le] + cnt[le]:off[le + 1]] == -1).all()
        assert off[le] % 16 == 0
    for t in range(T):
        for k in range(K):
            r = p["token_row"][t, k]
            assert (r >= 0) == (16 <= idx[t, k] < 48)
            if r >= 0:
                assert p["row_token"][r] == t and p["row_k"][r] == k


def _direct_dense_reference(inp, geo, offset, rsf):
    """Independent restatement: dense over all local experts with a routing mask."""
    import oracle

    idx, w = oracle.route(inp["routing_logits"], inp["routing_bias"], geo.n_group,
                          geo.topk_group, geo.top_k, rsf)
    a = oracle.dequant_act(inp["hidden_states"], inp["hidden_states_scale"])
    out = torch.zeros(a.shape[0], geo.hidden)
    for le in range(geo.num_local):
        w13 = oracle.dequant_weight(inp["gemm1_weights"][le], inp["gemm1_weights_scale"][le])
        w2 = oracle.dequant_weight(inp["gemm2_weights"][le], inp["gemm2_weights_scale"][le])
        g1 = a @ w13.t()
        x1, x2 = g1[:, :geo.inter], g1[:, geo.inter:]
        o = (x1 * torch.nn.functional.silu(x2)) @ w2.t()
        coef = torch.from_numpy(((idx == le + offset) * w).sum(1)).unsqueeze(1)
        out += coef * o
    return out


def test_moe_forward_matches_dense_restatement(oracle_mod):
    geo = W.TINY
    inp = W.make_inputs(geo, 24, seed=11)
    out = oracle_mod.moe_forward(*W.operator_args(inp), 0, 2.5, geo.n_group, geo.topk_group,
                                 geo.top_k)
    ref = _direct_dense_reference(inp, geo, 0, 2.5)
    torch.testing.assert_close(out.float(), ref, atol=1e-3, rtol=1e-2)
    assert out.dtype == torch.bfloat16 and out.shape == (24, geo.hidden)


def test_moe_forward_local_slice(oracle_mod):
    """Only experts inside [offset, offset + E_local) contribute (kernel.cu:857-859)."""
    geo = W.Geometry(hidden=256, inter=128, num_experts=16, num_local=8, n_group=4,
                     topk_group=2, top_k=4)
    inp = W.make_inputs(geo, 20, seed=5)
    out = oracle_mod.moe_forward(*W.operator_args(inp), 8, 2.5, 4, 2, 4)
    ref = _direct_dense_reference(inp, geo, 8, 2.5)
    torch.testing.assert_close(out.float(), ref, atol=1e-3, rtol=1e-2)


def test_quantisers_roundtrip():
    x = torch.randn(8, 256)
    q, s = W.quantize_rows_128(x)
    assert s.shape == (2, 8)
    deq = q.float() * s.t().repeat_interleave(128, 1)
    assert (deq - x).abs().max() <= 0.07 * x.abs().max()
    w = torch.randn(256, 384) * 0.02
    qw, sw = W.quantize_blocks_128(w)
    assert sw.shape == (2, 3)
    assert qw.float().abs().max() <= 448.0
