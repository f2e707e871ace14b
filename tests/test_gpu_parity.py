"""GPU parity of the sm_100a path against the CPU oracle, called through the C ABI.

* routing: indices and weights bit-exact (random, wide-range, tie-heavy and non-finite
  inputs; both geometries);
* permutation: expert counts, 16-row aligned offsets and the row maps bit-exact;
* whole operator: bf16 output within atol 2e-2 / rtol 2e-2
  and a relative-rms bound of 1e-2, at the tiny geometry and DeepSeek-V3 shapes;
* full sizes: sampled tokens against the oracle on those tokens only (each token's
  output depends only on its own routing and hidden state), run-to-run bit stability,
  and exact scaling in routed_scaling_factor.
"""
import numpy as np
import pytest
import torch

from fmoe_b200 import workloads as W

pytestmark = pytest.mark.gpu

ATOL = 2e-2
RTOL = 2e-2
REL_RMS = 1e-2


def _route_inputs(geo, T, seed, kind):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(T, geo.num_experts, generator=g)
    bias = torch.randn(geo.num_experts, generator=g) * 0.1
    if kind == "wide":
        logits = logits * 40.0
    elif kind == "ties":
        logits = torch.round(logits * 2.0) / 2.0
        bias = torch.zeros_like(bias)
    elif kind == "special":
        flat = logits.view(-1)
        n = flat.numel()
        sel = torch.randperm(n, generator=g)[: max(1, n // 20)]
        vals = torch.tensor([float("nan"), float("inf"), float("-inf"), 1e30, -1e30])
        flat[sel] = vals[torch.arange(sel.numel()) % 5]
        bias[0] = float("-inf")
    return logits.float(), bias.to(torch.bfloat16)


@pytest.mark.parametrize("geo", [W.TINY, W.DSV3], ids=["tiny", "dsv3"])
@pytest.mark.parametrize("T", [1, 7, 64, 1000, 4096])
@pytest.mark.parametrize("kind", ["normal", "wide", "ties", "special"])
def test_route_bitexact(fmoe, oracle_mod, geo, T, kind):
    logits, bias = _route_inputs(geo, T, 1000 + T, kind)
    ng, kg, k = geo.n_group, geo.topk_group, geo.top_k
    idx_o, w_o = oracle_mod.route(logits, bias, ng, kg, k, 2.5)
    idx_g, w_g = fmoe.route(logits.cuda(), bias.cuda(), ng, kg, k, 2.5,
                            num_local_experts=geo.num_local)
    idx_g = idx_g.cpu().numpy()
    w_g = w_g.cpu().numpy()
    assert np.array_equal(idx_g, idx_o)
    assert np.array_equal(w_g.view(np.uint32), w_o.view(np.uint32))


# ----------------------------------------------------------------------------- operator
_CACHE = {}


def _weights(geo, seed):
    key = (geo, seed)
    if key not in _CACHE:
        wg = W.make_weights(geo, seed, device="cuda")
        wc = {k: v.cpu() for k, v in wg.items()}
        _CACHE[key] = (wg, wc, {})
    return _CACHE[key]


def _inputs(geo, T, seed, skew_hot=0, offset=0):
    wg, wc, cache = _weights(geo, seed)
    acts = W.make_activations(geo, T, seed + 17 * T, device="cpu", skew_hot=skew_hot,
                              local_expert_offset=offset)
    gpu = {k: v.cuda() for k, v in acts.items() if isinstance(v, torch.Tensor)}
    gpu.update(wg)
    cpu = dict(acts)
    cpu.update(wc)
    return gpu, cpu, cache


def _oracle(oracle_mod, geo, cpu, offset, rsf, cache, tokens=None):
    args = W.operator_args(cpu)
    if tokens is not None:
        tok = torch.as_tensor(tokens)
        args[0] = args[0][tok]
        args[2] = args[2][tok]
        args[3] = args[3][:, tok].contiguous()
    return oracle_mod.moe_forward(*args, offset, rsf, geo.n_group, geo.topk_group, geo.top_k,
                                  weight_cache=cache)


def _check(out, ref):
    out = out.float().cpu()
    ref = ref.float().cpu()
    assert torch.isfinite(out).all()
    torch.testing.assert_close(out, ref, atol=ATOL, rtol=RTOL)
    den = ref.pow(2).mean().sqrt().clamp_min(1e-12)
    rel = (out - ref).pow(2).mean().sqrt() / den
    assert rel < REL_RMS, f"relative rms error {rel:.3e}"
    return float(rel)


def _run(fmoe, geo, gpu, offset, rsf, tile_n=0):
    out = fmoe.kernel(*W.operator_args(gpu), offset, rsf, tile_n=tile_n,
                      routing=(geo.n_group, geo.topk_group, geo.top_k))
    torch.cuda.synchronize()
    return out


def _device_error(fmoe, geo, T, offset=0, tile_n=0):
    prob = fmoe.make_problem(T, geo.num_experts, geo.num_local, geo.hidden, geo.inter, offset,
                             2.5, geo.n_group, geo.topk_group, geo.top_k, tile_n)
    ws = fmoe.Workspace.get(torch.device("cuda", torch.cuda.current_device()),
                            fmoe.workspace_bytes(prob))
    return fmoe.read_device_error(prob, ws)


TINY_LOCAL = W.Geometry(hidden=256, inter=128, num_experts=16, num_local=8, n_group=4,
                        topk_group=2, top_k=4)


@pytest.mark.parametrize("T", [1, 2, 16, 33, 100, 600])
@pytest.mark.parametrize("geo,offset", [(W.TINY, 0), (TINY_LOCAL, 8), (TINY_LOCAL, 0)],
                         ids=["tiny", "tiny_slice8", "tiny_slice0"])
def test_forward_tiny(fmoe, oracle_mod, T, geo, offset):
    gpu, cpu, cache = _inputs(geo, T, seed=1)
    out = _run(fmoe, geo, gpu, offset, 2.5)
    _check(out, _oracle(oracle_mod, geo, cpu, offset, 2.5, cache))
    assert _device_error(fmoe, geo, T, offset) == 0


@pytest.mark.parametrize("T", [1, 4, 16, 64])
def test_forward_dsv3_decode(fmoe, oracle_mod, T):
    geo = W.DSV3
    gpu, cpu, cache = _inputs(geo, T, seed=2)
    out = _run(fmoe, geo, gpu, 0, 2.5)
    _check(out, _oracle(oracle_mod, geo, cpu, 0, 2.5, cache))
    assert _device_error(fmoe, geo, T) == 0


@pytest.mark.parametrize("tile_n", [16, 32, 64, 128])
def test_forward_dsv3_every_tile(fmoe, oracle_mod, tile_n):
    geo = W.DSV3
    T = 200
    gpu, cpu, cache = _inputs(geo, T, seed=2)
    out = _run(fmoe, geo, gpu, 0, 2.5, tile_n=tile_n)
    _check(out, _oracle(oracle_mod, geo, cpu, 0, 2.5, cache))
    assert _device_error(fmoe, geo, T, tile_n=tile_n) == 0


# tile 0 = the autotune table (decode family up to 768 tokens, throughput family above);
# the explicit tiles force the other family on the same inputs
@pytest.mark.parametrize("T,skew,tile", [(512, 0, 0), (4096, 0, 0), (8192, 0, 0), (4096, 8, 0),
                                         (4096, 0, 64), (4096, 8, 64), (1024, 0, 128)],
                         ids=["T512", "T4096", "T8192", "T4096_skew", "T4096_tile64",
                              "T4096_skew_tile64", "T1024_tile128"])
def test_forward_dsv3_large_sampled(fmoe, oracle_mod, T, skew, tile):
    geo = W.DSV3
    gpu, cpu, cache = _inputs(geo, T, seed=2, skew_hot=skew)
    out = _run(fmoe, geo, gpu, 0, 2.5, tile_n=tile)
    g = torch.Generator().manual_seed(T + skew)
    tokens = torch.randperm(T, generator=g)[:48].sort().values
    ref = _oracle(oracle_mod, geo, cpu, 0, 2.5, cache, tokens=tokens)
    _check(out[tokens.cuda()], ref)
    assert _device_error(fmoe, geo, T, tile_n=tile) == 0


@pytest.mark.parametrize("T", [1, 16, 33, 100])
@pytest.mark.parametrize("geo,offset", [(W.TINY, 0), (TINY_LOCAL, 8)], ids=["tiny", "tiny_slice8"])
def test_forward_tiny_throughput_family(fmoe, oracle_mod, T, geo, offset):
    """tile_n 128: 128 token rows per MMA tile, partly empty at these sizes."""
    gpu, cpu, cache = _inputs(geo, T, seed=3)
    out = _run(fmoe, geo, gpu, offset, 2.5, tile_n=128)
    _check(out, _oracle(oracle_mod, geo, cpu, offset, 2.5, cache))
    assert _device_error(fmoe, geo, T, offset, tile_n=128) == 0


@pytest.mark.parametrize("T", [20011, 8192, 777, 64, 17, 1])
def test_plan_bitexact(fmoe, oracle_mod, T):
    """The permutation plan (expert counts and offsets, row <-> token maps) bit for bit against
    the oracle. The large T cases give the routing kernel's last CTA several batches of
    per-CTA counts per warp (512 and 1,251 CTAs), the last one partial."""
    geo = W.DSV3
    gpu, cpu, _ = _inputs(geo, T, seed=4)
    _run(fmoe, geo, gpu, 0, 2.5)
    prob = fmoe.make_problem(T, geo.num_experts, geo.num_local, geo.hidden, geo.inter, 0, 2.5)
    ws = fmoe.Workspace.get(torch.device("cuda", 0), fmoe.workspace_bytes(prob))
    view = fmoe.plan_view(prob, ws)
    idx_o, _ = oracle_mod.route(cpu["routing_logits"], cpu["routing_bias"], 8, 4, 8, 2.5)
    plan = oracle_mod.plan(idx_o, geo.num_local, 0, view["row_cap"])
    assert np.array_equal(view["expert_cnt"].cpu().numpy(), plan["expert_cnt"])
    assert np.array_equal(view["expert_off"].cpu().numpy(), plan["expert_off"])
    total = plan["total"]
    assert np.array_equal(view["row_token"].cpu().numpy()[:total], plan["row_token"][:total])
    assert np.array_equal(view["token_row"].cpu().numpy(), plan["token_row"].ravel())
    assert int(view["meta"][1]) == total


@pytest.mark.parametrize("T", [1, 5, 64, 300])
def test_operator_equals_route_then_routed_entry_point(fmoe, T):
    """fmoe_forward == fmoe_route followed by fmoe_forward_routed on the same routing
    (the expert-parallel layer's local step), bit for bit."""
    geo = W.DSV3
    gpu, _, _ = _inputs(geo, T, seed=9)
    out = _run(fmoe, geo, gpu, 0, 2.5)
    idx, w = fmoe.route(gpu["routing_logits"], gpu["routing_bias"], 8, 4, 8, 2.5,
                        num_local_experts=geo.num_local)
    routed = fmoe.forward_routed(idx, w, gpu["hidden_states"], gpu["hidden_states_scale"],
                                 gpu["gemm1_weights"], gpu["gemm1_weights_scale"],
                                 gpu["gemm2_weights"], gpu["gemm2_weights_scale"], 0,
                                 geo.num_experts, n_group=8, topk_group=4)
    torch.cuda.synchronize()
    assert torch.equal(out, routed)


def test_deterministic_and_rsf_scaling(fmoe):
    geo = W.DSV3
    T = 1024
    gpu, _, _ = _inputs(geo, T, seed=5)
    a = _run(fmoe, geo, gpu, 0, 2.5)
    b = _run(fmoe, geo, gpu, 0, 2.5)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    c = _run(fmoe, geo, gpu, 0, 5.0)
    assert torch.equal(c.float(), 2.0 * a.float())


def test_empty_batch(fmoe):
    geo = W.DSV3
    gpu, _, _ = _inputs(geo, 1, seed=2)
    args = W.operator_args(gpu)
    args[0] = args[0][:0]
    args[2] = args[2][:0]
    args[3] = args[3][:, :0].contiguous()
    out = fmoe.kernel(*args, 0, 2.5)
    assert out.shape == (0, geo.hidden)


def test_errors_mirror_reference(fmoe):
    geo = W.TINY
    gpu, _, _ = _inputs(geo, 4, seed=1)
    args = W.operator_args(gpu)
    bad = list(args)
    bad[0] = args[0].to(torch.float16)
    with pytest.raises(TypeError, match="dtype mismatch"):
        fmoe.kernel(*bad, 0, 2.5)
    bad = list(args)
    bad[2] = args[2].t().contiguous().t()
    with pytest.raises(ValueError):
        fmoe.kernel(*bad, 0, 2.5)
    bad = list(args)
    bad[3] = args[3].t().contiguous()
    with pytest.raises(ValueError, match="shape mismatch"):
        fmoe.kernel(*bad, 0, 2.5)


def test_tvm_ffi_binding_matches(fmoe):
    geo = W.DSV3
    gpu, _, _ = _inputs(geo, 64, seed=2)
    ref = _run(fmoe, geo, gpu, 0, 2.5)
    kern = fmoe.load_tvm_ffi_kernel()
    out = kern(*W.operator_args(gpu), 0, 2.5)
    out = torch.from_dlpack(out)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


# ----------------------------------------------------------------------------- reference
REF_SO = __import__("pathlib").Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "ref_kernel.so"


@pytest.fixture(scope="module")
def ref_kernel():
    """The reference operator itself (solution/cuda/kernel.cu, built by oracle/build_ref.sh)."""
    if not REF_SO.exists():
        pytest.skip("reference kernel not built (oracle/build_ref.sh)")
    import tvm_ffi

    return tvm_ffi.load_module(str(REF_SO))["kernel"]


@pytest.mark.parametrize("T", [1, 16, 64, 600])
def test_oracle_pinned_to_reference_kernel(ref_kernel, oracle_mod, T):
    """Pins the CPU oracle against the reference's own CUDA implementation (DS-V3 shapes,
    both of its paths: device-only for T <= 512, grouped CUTLASS for T > 512)."""
    geo = W.DSV3
    gpu, cpu, cache = _inputs(geo, T, seed=2)
    ref_out = torch.from_dlpack(ref_kernel(*W.operator_args(gpu), 0, 2.5))
    torch.cuda.synchronize()
    _check(ref_out, _oracle(oracle_mod, geo, cpu, 0, 2.5, cache))


@pytest.mark.parametrize("T", [4, 256, 1024])
def test_matches_reference_kernel(fmoe, ref_kernel, T):
    geo = W.DSV3
    gpu, _, _ = _inputs(geo, T, seed=6)
    ref_out = torch.from_dlpack(ref_kernel(*W.operator_args(gpu), 0, 2.5))
    out = _run(fmoe, geo, gpu, 0, 2.5)
    _check(out, ref_out)


@pytest.mark.parametrize("T", [1, 64, 2048])
def test_cuda_graph_replay_matches_eager(fmoe, T):
    """The operator is capturable (no host sync, no allocation inside the call) and a
    graph replay (memset + five PDL-linked kernels) gives the eager result bit for bit."""
    geo = W.DSV3
    gpu, _, _ = _inputs(geo, T, seed=2)
    args = W.operator_args(gpu)
    ref = _run(fmoe, geo, gpu, 0, 2.5)
    out = torch.empty_like(ref)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fmoe.kernel(*args, 0, 2.5, out=out)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fmoe.kernel(*args, 0, 2.5, out=out)
    out.zero_()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    del graph


@pytest.mark.parametrize("T", [16, 64])
def test_library_graph_cache_replays_and_reads_current_inputs(fmoe, T):
    """fmoe_forward replays repeated calls from a cached CUDA graph: the replays match the
    eager first call bit for bit, and new input contents behind the same pointers are
    read (the graph freezes addresses, not data)."""
    geo = W.DSV3
    gpu, _, _ = _inputs(geo, T, seed=7)
    args = W.operator_args(gpu)
    out = torch.empty(T, geo.hidden, dtype=torch.bfloat16, device="cuda")
    fmoe.kernel(*args, 0, 2.5, out=out)  # first sighting: eager
    torch.cuda.synchronize()
    ref = out.clone()
    for _ in range(3):  # second sighting captures, then replays
        out.zero_()
        fmoe.kernel(*args, 0, 2.5, out=out)
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    # new routing logits and activations in the same buffers
    g = torch.Generator().manual_seed(99)
    gpu["routing_logits"].copy_(torch.randn(gpu["routing_logits"].shape, generator=g))
    gpu["hidden_states"].copy_(gpu["hidden_states"].flip(0))
    fmoe.kernel(*args, 0, 2.5, out=out)
    fresh = torch.empty_like(out)
    fmoe.kernel(*args, 0, 2.5, out=fresh)  # different output pointer: a new key, eager
    torch.cuda.synchronize()
    assert not torch.equal(out.view(torch.int16), ref.view(torch.int16))
    assert torch.equal(out.view(torch.int16), fresh.view(torch.int16))


# ----------------------------------------------------------------------------- weight pre-layout
def _prelayout_numpy(w13, w2, I):
    """Restatement of fmoe_prelayout_weights: every (expert, row tile, 128-K step) weight tile
    as 256 rows x 128 bytes with 16-byte chunk c of row r stored at chunk c ^ (r % 8)."""
    E, _, H = w13.shape
    tiles1, tiles2 = [], []
    perm = np.array([[c ^ (r & 7) for c in range(8)] for r in range(256)])

    def image(rows):  # rows: [256, 128] uint8
        out = np.empty_like(rows)
        for r in range(256):
            chunks = rows[r].reshape(8, 16)
            out[r].reshape(8, 16)[perm[r]] = chunks
        return out

    for e in range(E):
        for m in range(I // 128):
            for k in range(H // 128):
                g = w13[e, 128 * m:128 * m + 128, 128 * k:128 * k + 128]
                u = w13[e, I + 128 * m:I + 128 * m + 128, 128 * k:128 * k + 128]
                tiles1.append(image(np.concatenate([g, u])))
        for m in range(H // 256):
            for k in range(I // 128):
                tiles2.append(image(w2[e, 256 * m:256 * m + 256, 128 * k:128 * k + 128]))
    return np.concatenate(tiles1).ravel(), np.concatenate(tiles2).ravel()


def test_prelayout_matches_restatement(fmoe):
    geo = W.TINY  # H = 256, I = 128: 2 GEMM1 tiles and 2 GEMM2 tiles per expert
    gpu, cpu, _ = _inputs(geo, 4, seed=8)
    w13p, w2p = fmoe.prelayout_weights(gpu["gemm1_weights"], gpu["gemm2_weights"])
    torch.cuda.synchronize()
    e1, e2 = _prelayout_numpy(cpu["gemm1_weights"].view(torch.uint8).numpy(),
                              cpu["gemm2_weights"].view(torch.uint8).numpy(), geo.inter)
    assert np.array_equal(w13p.view(torch.uint8).cpu().numpy().ravel(), e1)
    assert np.array_equal(w2p.view(torch.uint8).cpu().numpy().ravel(), e2)


@pytest.mark.parametrize("T,skew,tile", [(1, 0, 0), (64, 0, 0), (200, 0, 64), (200, 0, 32),
                                         (1024, 0, 128), (4096, 8, 0)])
def test_prelaid_weights_same_bits(fmoe, T, skew, tile):
    """Both GEMM families fed from pre-laid-out weights (one bulk copy per weight tile) give
    the output of the tensor-map path bit for bit: the shared-memory images are the same."""
    geo = W.DSV3
    gpu, _, _ = _inputs(geo, T, seed=6, skew_hot=skew)
    w13p, w2p = fmoe.prelayout_weights(gpu["gemm1_weights"], gpu["gemm2_weights"])
    args = W.operator_args(gpu)
    ref = fmoe.kernel(*args, 0, 2.5, tile_n=tile)
    args[4], args[6] = w13p, w2p
    out = fmoe.kernel(*args, 0, 2.5, tile_n=tile, prelaid=True)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    if T == 64:
        idx, w = fmoe.route(gpu["routing_logits"], gpu["routing_bias"], 8, 4, 8, 2.5,
                            num_local_experts=geo.num_local)
        routed = fmoe.forward_routed(idx, w, gpu["hidden_states"], gpu["hidden_states_scale"],
                                     w13p, gpu["gemm1_weights_scale"], w2p,
                                     gpu["gemm2_weights_scale"], 0, geo.num_experts, n_group=8,
                                     topk_group=4, prelaid=True)
        torch.cuda.synchronize()
        assert torch.equal(routed, ref)
