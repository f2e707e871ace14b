"""Expert-parallel layer: host-side exchange logic on CPU ranks (gloo).

The routing and the per-rank expert compute are the CPU oracle, so these tests check the
dispatch / combine logic of fmoe_b200.ep (destination masks, ordering, all-to-all-v,
unpacking, rank-ordered reduction) against the oracle's single-process full layer, on 2
and 4 ranks. A failure test kills one rank before the exchange and checks that the other
rank gets an error from its collective within the process-group timeout instead of
waiting forever.
"""
import datetime
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent
for _p in (ROOT, ROOT / "fused-moe-yws_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

GEO_E, GEO_H, GEO_I, NG, KG, K = 16, 256, 128, 4, 2, 4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _geo():
    from fmoe_b200 import workloads as W

    return W.Geometry(hidden=GEO_H, inter=GEO_I, num_experts=GEO_E, num_local=GEO_E,
                      n_group=NG, topk_group=KG, top_k=K)


def _ep_worker(rank, world, port, T, result_q, placement_mode=None):
    import oracle
    from fmoe_b200 import ep
    from fmoe_b200 import workloads as W

    _init(rank, world, port)
    torch.set_num_threads(1)
    geo = _geo()
    full = W.make_weights(geo, seed=9, device="cpu")
    per = GEO_E // world
    acts = W.make_activations(geo, T + rank, seed=100 + rank, device="cpu")

    def route_fn(logits, bias):
        idx, w = oracle.route(logits, bias, NG, KG, K, 2.5)
        return torch.from_numpy(idx), torch.from_numpy(w)

    placement = None
    if placement_mode == "shuffle":
        placement = torch.randperm(GEO_E, generator=torch.Generator().manual_seed(5)).tolist()
    elif placement_mode in ("calibrated", "local"):
        cal = W.make_activations(geo, 64, seed=700 + rank, device="cpu")
        placement = ep.calibrate_placement(route_fn, cal["routing_logits"], acts["routing_bias"],
                                           GEO_E, mode="local" if placement_mode == "local"
                                           else "balanced")
        allp = [None] * world
        dist.all_gather_object(allp, placement)
        assert all(p == placement for p in allp)
    mine = placement[rank * per:(rank + 1) * per] if placement else list(range(rank * per, (rank + 1) * per))
    local = {k: v[mine].contiguous() for k, v in full.items()}

    def local_fn(idx, w, hs, sc, offset):
        return oracle.moe_forward_routed(idx, w, hs, sc, local["gemm1_weights"],
                                         local["gemm1_weights_scale"], local["gemm2_weights"],
                                         local["gemm2_weights_scale"], offset)

    layer = ep.ExpertParallelMoE(num_experts=GEO_E, n_group=NG, topk_group=KG, top_k=K,
                                 routed_scaling_factor=2.5, route_fn=route_fn,
                                 local_fn=local_fn, placement=placement)
    assert layer.local_experts() == mine
    out = layer.forward(acts["routing_logits"], acts["routing_bias"], acts["hidden_states"],
                        acts["hidden_states_scale"])
    ref = oracle.moe_forward(*W.operator_args({**acts, **full}), 0, 2.5, NG, KG, K)
    err = (out.float() - ref.float()).abs()
    rel = float((out.float() - ref.float()).norm() / ref.float().norm().clamp_min(1e-12))
    ok = bool((err <= 2e-2 + 2e-2 * ref.float().abs()).all())
    result_q.put((rank, ok, rel, tuple(out.shape)))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,placement_mode", [(2, None), (4, None), (2, "shuffle"),
                                                  (4, "calibrated"), (4, "local")])
def test_ep_matches_full_layer(world, placement_mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, world, port, 24, q, placement_mode))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok, rel, shape in sorted(results):
        assert shape == (24 + rank, GEO_H)
        assert ok and rel < 1e-2, (rank, rel)


def test_balanced_placement():
    from fmoe_b200 import ep

    g = torch.Generator().manual_seed(3)
    rows = (torch.rand(256, generator=g) ** 4 * 2000).to(torch.int64)  # skewed loads
    rows[:10] = 0
    for world in (1, 2, 4, 8):
        pl = ep.balanced_placement(rows, world)
        assert sorted(pl) == list(range(256))
        per = 256 // world
        cost = ep.placement_cost(rows)
        work = [int(cost[pl[r * per:(r + 1) * per]].sum()) for r in range(world)]
        contig = [int(cost[r * per:(r + 1) * per].sum()) for r in range(world)]
        assert max(work) <= max(contig)
        assert max(work) - min(work) <= int(cost.max())  # LPT bound on the spread
        assert pl == ep.balanced_placement(rows.tolist(), world)  # deterministic
    with pytest.raises(ValueError):
        ep.balanced_placement(rows[:255], 2)


def _skewed_routing(T, E, K, seed):
    g = torch.Generator().manual_seed(seed)
    pop = torch.rand(E, generator=g) ** 3 + 0.02  # skewed expert popularity
    idx = torch.stack([torch.multinomial(pop, K, replacement=False, generator=g)
                       for _ in range(T)]).to(torch.int32)
    idx[torch.rand(T, K, generator=g) < 0.02] = -1  # a few unselected slots
    return idx


def _rank_costs(idx, placement, world, recv_cost):
    import numpy as np

    E = len(placement)
    per = E // world
    owner = np.zeros(E, dtype=np.int64)
    for i, e in enumerate(placement):
        owner[e] = i // per
    ids = idx.numpy()
    valid = ids >= 0
    rows = np.bincount(ids[valid], minlength=E)
    tiles = np.array([((rows[owner == r] + 127) // 128).sum() for r in range(world)])
    recv = np.zeros(world)
    for t in range(ids.shape[0]):
        for r in set(owner[ids[t][valid[t]]].tolist()):
            recv[r] += 1
    return tiles + recv_cost * recv


def test_locality_placement():
    from fmoe_b200 import ep

    E, K = 64, 4
    idx = _skewed_routing(1500, E, K, seed=7)
    assert ep.locality_placement(idx, E, 1) == list(range(E))
    for world in (2, 4, 8):
        for search in ("pairs", "max-rank"):
            pl = ep.locality_placement(idx, E, world, search=search)
            assert sorted(pl) == list(range(E))
            assert pl == ep.locality_placement(idx.clone(), E, world, search=search)
            rc = ep.RECV_TOKEN_COST_IN_TILES
            local = _rank_costs(idx, pl, world, rc)
            contig = _rank_costs(idx, list(range(E)), world, rc)
            assert local.max() <= contig.max() + 1e-9
    with pytest.raises(ValueError):
        ep.locality_placement(idx, 63, 2)


def test_placement_validation():
    from fmoe_b200 import ep

    with pytest.raises(ValueError):
        ep.ExpertParallelMoE(num_experts=16, n_group=4, topk_group=2, top_k=4,
                             placement=list(range(15)) + [0])
    layer = ep.ExpertParallelMoE(num_experts=16, n_group=4, topk_group=2, top_k=4,
                                 placement=list(range(16)))
    assert layer.placement is None and layer.local_experts() == list(range(16))
    layer = ep.ExpertParallelMoE(num_experts=16, n_group=4, topk_group=2, top_k=4,
                                 placement=list(reversed(range(16))))
    idx = torch.tensor([[0, 15, -1, 3]], dtype=torch.int32)
    assert layer.place_ids(idx).tolist() == [[15, 0, -1, 12]]


def test_pack_unpack_roundtrip():
    from fmoe_b200 import ep
    from fmoe_b200 import workloads as W

    acts = W.make_activations(_geo(), 10, seed=3)
    idx = torch.randint(0, GEO_E, (10, K), dtype=torch.int32)
    w = torch.rand(10, K)
    tokens = torch.tensor([7, 1, 3])
    buf = ep.pack_rows(acts["hidden_states"], acts["hidden_states_scale"], idx, w, tokens)
    hs, sc, ii, ww = ep.unpack_rows(buf, GEO_H, K)
    assert torch.equal(hs.view(torch.uint8), acts["hidden_states"].view(torch.uint8)[tokens])
    assert torch.equal(sc, acts["hidden_states_scale"][:, tokens])
    assert torch.equal(ii, idx[tokens]) and torch.equal(ww, w[tokens])


def _dying_worker(rank, world, port, result_q):
    from fmoe_b200 import workloads as W
    from fmoe_b200 import ep

    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        os._exit(3)  # the rank dies between steps, before the exchange
    geo = _geo()
    acts = W.make_activations(geo, 8, seed=1)

    def route_fn(logits, bias):
        idx = torch.zeros(logits.shape[0], K, dtype=torch.int32)
        idx[:, 1] = GEO_E - 1  # one route on the peer's experts
        return idx, torch.ones(logits.shape[0], K)

    layer = ep.ExpertParallelMoE(num_experts=GEO_E, n_group=NG, topk_group=KG, top_k=K,
                                 route_fn=route_fn, local_fn=lambda *a: None)
    try:
        layer.forward(acts["routing_logits"], acts["routing_bias"], acts["hidden_states"],
                      acts["hidden_states_scale"])
        result_q.put((rank, "no error"))
    except Exception as e:  # the collective must fail, not hang
        result_q.put((rank, type(e).__name__))


def test_ep_peer_failure_is_reported():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank, what = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert rank == 0 and what != "no error"
