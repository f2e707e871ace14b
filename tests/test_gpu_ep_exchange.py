"""The expert-parallel exchange kernels (fmoe_ep_plan / pack / unpack / combine) on one B200,
bit for bit against the framework-op restatement in fmoe_b200/ep.py that the gloo CPU tests
exercise, plus the whole layer with the exchange kernels on and off (world size 1)."""
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
for _p in (ROOT, ROOT / "fused-moe-yws_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

pytestmark = pytest.mark.gpu


def _routing(T, K, E, world, seed, drop=0.1):
    g = torch.Generator().manual_seed(seed)
    if T == 0:
        return (torch.empty(0, K, dtype=torch.int32, device="cuda"),
                torch.empty(0, K, dtype=torch.float32, device="cuda"))
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32)
    idx[torch.rand(T, K, generator=g) < drop] = -1  # unselected slots
    w = torch.rand(T, K, generator=g)
    return idx.cuda(), w.cuda()


def _torch_plan(idx, world, e_per_rank):
    T, K = idx.shape
    owner = torch.where(idx >= 0, idx // e_per_rank, torch.full_like(idx, -1))
    mask = torch.zeros(T, world, dtype=torch.bool, device=idx.device)
    valid = owner >= 0
    rows = torch.arange(T, device=idx.device).unsqueeze(1).expand(T, K)
    mask[rows[valid], owner[valid].long()] = True
    order = torch.nonzero(mask.t(), as_tuple=False)
    return mask.sum(0), order[:, 1], mask


@pytest.mark.parametrize("T,world", [(1, 1), (37, 2), (1500, 4), (4096, 8), (0, 2)])
def test_plan_matches_restatement(T, world):
    import fmoe_b200

    E, K = 256, 8
    idx, _ = _routing(T, K, E, world, seed=T + world)
    pos, tokens, counts = fmoe_b200.ep_plan(idx, world, E // world)
    cnt_ref, tok_ref, mask = _torch_plan(idx, world, E // world)
    assert counts.tolist() == cnt_ref.tolist()
    n = int(cnt_ref.sum())
    assert torch.equal(tokens[:n].long(), tok_ref)
    # pos[d, t] is the row of t in d's segment, -1 where t does not go to d
    base = torch.cumsum(cnt_ref, 0) - cnt_ref
    for d in range(world):
        sel = mask[:, d]
        expect = torch.full((T,), -1, dtype=torch.int64, device=idx.device)
        expect[sel] = base[d] + torch.arange(int(sel.sum()), device=idx.device)
        assert torch.equal(pos[d].long(), expect)


@pytest.mark.parametrize("T,world", [(1, 2), (1500, 4), (4096, 8), (0, 2)])
def test_placed_plan_equals_plan_of_mapped_ids(T, world):
    """fmoe_ep_plan_placed: ids replaced in place by their placement positions (ids < 0
    kept), then the same plan as fmoe_ep_plan of the mapped ids."""
    import fmoe_b200
    from fmoe_b200 import ep

    E, K = 256, 8
    idx, _ = _routing(T, K, E, world, seed=7 * T + world)
    rows = torch.bincount(idx[idx >= 0].long().cpu(), minlength=E)
    layer = ep.ExpertParallelMoE(num_experts=E, placement=ep.balanced_placement(rows, world)
                                 if T else list(reversed(range(E))))
    mapped = layer.place_ids(idx)
    got = idx.clone()
    pos, tokens, counts = fmoe_b200.ep_plan(got, world, E // world, layer._dev_pos(idx.device))
    assert torch.equal(got, mapped)
    pos_r, tokens_r, counts_r = fmoe_b200.ep_plan(mapped.clone(), world, E // world)
    assert torch.equal(counts, counts_r)
    n = int(counts_r.sum())
    assert torch.equal(tokens[:n], tokens_r[:n]) and torch.equal(pos, pos_r)


@pytest.mark.parametrize("H,K,T,world", [(7168, 8, 300, 4), (256, 4, 33, 2)])
def test_pack_unpack_match_restatement(H, K, T, world):
    import fmoe_b200
    from fmoe_b200 import ep

    E = 256 if K == 8 else 16
    idx, w = _routing(T, K, E, world, seed=H + T)
    g = torch.Generator().manual_seed(3)
    hs = (torch.randn(T, H, generator=g) * 4).to(torch.float8_e4m3fn).cuda()
    sc = torch.rand(H // 128, T, generator=g).cuda()
    pos, tokens, counts = fmoe_b200.ep_plan(idx, world, E // world)
    n = int(counts.sum())
    send = fmoe_b200.ep_pack(hs, sc, idx, w, pos, n)
    ref = ep.pack_rows(hs, sc, idx, w, tokens[:n].long())
    assert torch.equal(send, ref)
    hs_r, sc_r, idx_r, w_r = fmoe_b200.ep_unpack(send, H, K)
    r_hs, r_sc, r_idx, r_w = ep.unpack_rows(ref, H, K)
    assert torch.equal(hs_r.view(torch.uint8), r_hs.view(torch.uint8))
    assert torch.equal(sc_r, r_sc) and torch.equal(idx_r, r_idx) and torch.equal(w_r, r_w)


@pytest.mark.parametrize("T,world", [(513, 4), (64, 8), (5, 1)])
def test_combine_matches_rank_ordered_index_add(T, world):
    import fmoe_b200

    H, K, E = 7168, 8, 256
    idx, _ = _routing(T, K, E, world, seed=11 * T)
    pos, tokens, counts = fmoe_b200.ep_plan(idx, world, E // world)
    n = int(counts.sum())
    g = torch.Generator().manual_seed(5)
    back = (torch.randn(n, H, generator=g) * 3).to(torch.bfloat16).cuda()
    out = fmoe_b200.ep_combine(back, pos, T)
    ref = torch.zeros(T, H, dtype=torch.float32, device="cuda")
    start = 0
    tok = tokens[:n].long()
    for c in counts.tolist():
        if c:
            ref.index_add_(0, tok[start:start + c], back[start:start + c].float())
        start += c
    assert torch.equal(out, ref.to(torch.bfloat16))


def test_layer_same_with_and_without_exchange_kernels():
    from fmoe_b200 import ep
    from fmoe_b200 import workloads as W

    geo = W.DSV3
    weights = W.make_expert_slice(geo, 7, 0, 256, device="cuda")
    acts = W.make_activations(geo, 96, 21, device="cuda")
    a4 = [acts[k] for k in W.OPERATOR_ARGS[:4]]
    fused = ep.ExpertParallelMoE(weights=weights, fused_exchange=True).forward(*a4)
    plain = ep.ExpertParallelMoE(weights=weights, fused_exchange=False).forward(*a4)
    torch.cuda.synchronize()
    assert torch.equal(fused, plain)
    # a placement (weights stacked in placement order) gives the same layer on one rank; the
    # bits can differ only where the expert order moves a row into a stream-K split tile
    pl = torch.randperm(256, generator=torch.Generator().manual_seed(4)).tolist()
    wp = {k: v[pl].contiguous() for k, v in weights.items()}
    placed = ep.ExpertParallelMoE(weights=wp, placement=pl).forward(*a4)
    placed_plain = ep.ExpertParallelMoE(weights=wp, placement=pl,
                                        fused_exchange=False).forward(*a4)
    torch.cuda.synchronize()
    assert torch.equal(placed, placed_plain)
    torch.testing.assert_close(placed.float(), fused.float(), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_offsets_match_host_arithmetic(world):
    """fmoe_ep_offsets against the host-side offset arithmetic of the P2P step."""
    import fmoe_b200

    g = torch.Generator().manual_seed(world)
    m = torch.randint(0, 500, (world, world + 1), generator=g, dtype=torch.int64)
    cnt = m[:, :world].tolist()
    for me in range(world):
        tables, rows = fmoe_b200.ep_offsets(m.cuda(), me)

        def src_start(d, s):
            return sum(cnt[q][d] for q in range(s))

        def seg_base(s, d):
            return sum(cnt[s][:d])

        starts = [src_start(me, s) for s in range(world + 1)]
        expect = ([src_start(d, me) - seg_base(me, d) for d in range(world)] + starts +
                  [seg_base(s, me) - starts[s] for s in range(world)])
        assert tables.tolist() == expect and rows.item() == starts[world]


def test_count_entry_points_match_exact_sizes():
    """fmoe_ep_unpack_count and fmoe_forward_routed_count on capacity-sized buffers give the
    first R rows exactly as fmoe_ep_unpack / fmoe_forward_routed on R rows."""
    import fmoe_b200
    from fmoe_b200 import workloads as W

    H, K, R, cap, EL = 7168, 8, 300, 512, 32
    row_bytes = fmoe_b200.ep_payload_bytes(H, K)
    g = torch.Generator().manual_seed(11)
    geo = W.DSV3
    acts = W.make_activations(geo, R, 5, device="cuda")
    idx, w = fmoe_b200.route(acts["routing_logits"], acts["routing_bias"], 8, 4, 8, 2.5)
    recv = torch.randint(0, 255, (cap, row_bytes), generator=g, dtype=torch.uint8).cuda()
    # real payload rows in front (valid FP8, scales, ids, weights)
    pos, _, counts = fmoe_b200.ep_plan(idx, 1, 256)
    recv[:R] = fmoe_b200.ep_pack(acts["hidden_states"], acts["hidden_states_scale"], idx, w,
                                 pos, R)
    rows = torch.tensor([R], dtype=torch.int32, device="cuda")
    hs_c, sc_c, idx_c, w_c = fmoe_b200.ep_unpack_count(recv, cap, rows, H, K)
    hs, sc, ii, ww = fmoe_b200.ep_unpack(recv[:R].contiguous(), H, K)
    assert torch.equal(hs_c[:R].view(torch.uint8), hs.view(torch.uint8))
    assert torch.equal(sc_c[:, :R], sc) and torch.equal(idx_c[:R], ii) and torch.equal(w_c[:R], ww)
    wts = W.make_expert_slice(geo, 3, 0, EL, device="cuda")
    wl = [wts[k] for k in W.OPERATOR_ARGS[4:]]
    # stale ids past R must not be routed: fill them with a local expert
    idx_c[R:] = 3
    exact = fmoe_b200.forward_routed(ii, ww, hs, sc, *wl, 0, 256)
    out = torch.full((cap, H), 7.0, dtype=torch.bfloat16, device="cuda")
    for _ in range(3):  # eager, then captured, then replayed from the library's graph cache
        got = fmoe_b200.forward_routed(idx_c, w_c, hs_c, sc_c, *wl, 0, 256, out=out,
                                       num_tokens_dev=rows)
        torch.cuda.synchronize()
        torch.testing.assert_close(got[:R].float(), exact.float(), atol=1e-2, rtol=1e-2)
        assert bool((got[R:] == 7.0).all())  # rows past the count untouched
    # the count is read at run time: a smaller count on the same buffers
    rows.fill_(100)
    got = fmoe_b200.forward_routed(idx_c, w_c, hs_c, sc_c, *wl, 0, 256, out=out,
                                   num_tokens_dev=rows)
    exact100 = fmoe_b200.forward_routed(ii[:100].contiguous(), ww[:100].contiguous(),
                                        hs[:100].contiguous(), sc[:, :100].contiguous(), *wl, 0,
                                        256)
    torch.cuda.synchronize()
    torch.testing.assert_close(got[:100].float(), exact100.float(), atol=1e-2, rtol=1e-2)
    assert fmoe_b200.poll_device_error() == 0


def test_operator_returns_rows_straight_to_sources():
    """fmoe_forward_routed_count_p2p: the combine writes row r of source s at row
    r + row_shift[s] of buffer s (here two local buffers stand in for two ranks' return
    buffers), bit-identical to the rows of the plain call; rows past the count and the
    rows of `out` are not written; a shift out of the capacity is flagged, not written."""
    import types
    import fmoe_b200
    from fmoe_b200 import workloads as W

    H, K, R, cap, EL = 7168, 8, 150, 256, 32
    geo = W.DSV3
    acts = W.make_activations(geo, R, 8, device="cuda")
    idx, w = fmoe_b200.route(acts["routing_logits"], acts["routing_bias"], 8, 4, 8, 2.5)
    wts = W.make_expert_slice(geo, 2, 0, EL, device="cuda")
    wl = [wts[k] for k in W.OPERATOR_ARGS[4:]]
    hs = torch.zeros(cap, H, dtype=torch.float8_e4m3fn, device="cuda")
    sc = torch.ones(H // 128, cap, dtype=torch.float32, device="cuda")
    ii = torch.full((cap, K), 1, dtype=torch.int32, device="cuda")
    ww = torch.zeros(cap, K, dtype=torch.float32, device="cuda")
    hs[:R] = acts["hidden_states"]
    sc[:, :R] = acts["hidden_states_scale"]
    ii[:R] = idx
    ww[:R] = w
    rows = torch.tensor([R], dtype=torch.int32, device="cuda")
    plain = fmoe_b200.forward_routed(ii, ww, hs, sc, *wl, 0, 256, num_tokens_dev=rows)
    bufs = [torch.full((cap, H), 3.0, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    peers = types.SimpleNamespace(back_ptrs=torch.tensor([b.data_ptr() for b in bufs],
                                                         dtype=torch.int64, device="cuda"))
    src_start = torch.tensor([0, 60, R], dtype=torch.int64, device="cuda")
    shift = torch.tensor([10, -60 + 7], dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.full((cap, H), 5.0, dtype=torch.bfloat16, device="cuda")
    for _ in range(3):  # eager, captured, replayed
        for b in bufs:
            b.fill_(3.0)
        fmoe_b200.forward_routed(ii, ww, hs, sc, *wl, 0, 256, num_tokens_dev=rows, out=out,
                                 return_to=(peers, src_start, shift, cap, err))
        torch.cuda.synchronize()
        assert torch.equal(bufs[0][10:70], plain[:60]) and torch.equal(bufs[1][7:97], plain[60:R])
        assert bool((bufs[0][:10] == 3.0).all()) and bool((bufs[0][70:] == 3.0).all())
        assert bool((bufs[1][:7] == 3.0).all()) and bool((bufs[1][97:] == 3.0).all())
        assert bool((out == 5.0).all()) and err.item() == 0
    shift[1] = cap  # every row of source 1 lands past the capacity
    bufs[1].fill_(3.0)
    fmoe_b200.forward_routed(ii, ww, hs, sc, *wl, 0, 256, num_tokens_dev=rows, out=out,
                             return_to=(peers, src_start, shift, cap, err))
    torch.cuda.synchronize()
    assert err.item() == 2 and bool((bufs[1] == 3.0).all())
    assert fmoe_b200.poll_device_error() == 0


def test_exchange_entry_points_reject_bad_arguments():
    import fmoe_b200

    lib = fmoe_b200.load_library()
    assert lib.fmoe_ep_plan(None, 4, 8, 2, 128, None, None, None, None) == fmoe_b200.FMOE_ERR_VALUE
    assert lib.fmoe_ep_plan_placed(None, 4, 8, 2, 128, None, 256, None, None, None,
                                   None) == fmoe_b200.FMOE_ERR_VALUE
    assert lib.fmoe_ep_offsets(None, 2, 0, None, None, None) == fmoe_b200.FMOE_ERR_VALUE
    assert lib.fmoe_ep_offsets(None, 2, 2, None, None, None) == fmoe_b200.FMOE_ERR_VALUE
    assert lib.fmoe_ep_unpack_count(None, 3, None, 7168, 8, None, None, None, None,
                                    None) == fmoe_b200.FMOE_ERR_VALUE
    assert lib.fmoe_ep_combine(None, None, 4, 7168, 0, None, None) == fmoe_b200.FMOE_ERR_VALUE
    assert lib.fmoe_ep_unpack(None, 3, 100, 8, None, None, None, None, None) == \
        fmoe_b200.FMOE_ERR_VALUE
