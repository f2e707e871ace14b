"""Seeded synthetic inputs for the fused MoE operator.

The contest workloads (FlashInfer-Bench dataset ``mlsys26-contest``) are not available
offline. These generators stand in for them with the shapes, dtypes and value
distributions the benchmark configurations name:

* ``routing_logits`` fp32 N(0, 1) ``[T, E_global]``
* ``routing_bias`` bf16 N(0, 0.1) ``[E_global]`` (skew: +3.0 on 8 hot experts inside the
  local slice)
* ``hidden_states`` N(0, 1) quantised to FP8 e4m3 with per-token, per-128-column fp32
  scales ``amax / 448``, stored transposed as ``[H / 128, T]``
* ``gemm1_weights`` ``[E_local, 2I, H]`` and ``gemm2_weights`` ``[E_local, H, I]``, both
  N(0, 0.02) quantised per 128x128 block with fp32 scales ``amax / 448``

Each expert's weights come from their own generator (seed, expert), so a CPU checker
can regenerate only the experts a test routes to. Random streams differ between
``cpu`` and ``cuda`` generators; tests that compare devices generate once and copy.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import torch

FP8_MAX = 448.0


@dataclass(frozen=True)
class Geometry:
    hidden: int            # H
    inter: int             # I
    num_experts: int       # E_global
    num_local: int         # E_local
    n_group: int
    topk_group: int
    top_k: int

    @property
    def kb_hidden(self) -> int:
        return self.hidden // 128


DSV3 = Geometry(hidden=7168, inter=2048, num_experts=256, num_local=32, n_group=8,
                topk_group=4, top_k=8)
TINY = Geometry(hidden=256, inter=128, num_experts=16, num_local=16, n_group=4,
                topk_group=2, top_k=4)

# Routing constants of the definition, keyed by the number of global experts (the
# operator signature carries no n_group / topk_group / top_k).
ROUTING_BY_EXPERTS = {256: (8, 4, 8), 16: (4, 2, 4)}


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed) & 0x7FFFFFFFFFFFFFFF)
    return g


def quantize_rows_128(x: torch.Tensor):
    """Per-row, per-128-column FP8 e4m3 quantisation. Returns (fp8 [T, H], scale [H/128, T])."""
    T, H = x.shape
    xb = x.view(T, H // 128, 128)
    amax = xb.abs().amax(-1)
    scale = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    q = (xb / scale.unsqueeze(-1)).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.view(T, H), scale.t().contiguous()


def quantize_blocks_128(w: torch.Tensor):
    """128x128-block FP8 e4m3 quantisation of one matrix [N, K] -> (fp8, scale [N/128, K/128])."""
    N, K = w.shape
    wb = w.view(N // 128, 128, K // 128, 128)
    amax = wb.abs().amax(dim=(1, 3))
    scale = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    q = (wb / scale[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.view(N, K), scale


def make_activations(geo: Geometry, T: int, seed: int, device="cpu", skew_hot: int = 0,
                     local_expert_offset: int = 0):
    """routing_logits, routing_bias, hidden_states, hidden_states_scale (+ hot expert ids)."""
    g = _gen(device, seed * 7919 + 1)
    logits = torch.randn(T, geo.num_experts, generator=g, device=device, dtype=torch.float32)
    bias = torch.randn(geo.num_experts, generator=g, device=device, dtype=torch.float32) * 0.1
    hot = []
    if skew_hot:
        perm = torch.randperm(geo.num_local, generator=_gen("cpu", seed * 7919 + 2))
        hot = sorted(int(local_expert_offset + p) for p in perm[:skew_hot])
        bias[hot] += 3.0
    bias = bias.to(torch.bfloat16)
    x = torch.randn(T, geo.hidden, generator=g, device=device, dtype=torch.float32)
    hs, hs_scale = quantize_rows_128(x)
    return dict(routing_logits=logits, routing_bias=bias, hidden_states=hs,
                hidden_states_scale=hs_scale, hot_experts=hot)


def make_expert(geo: Geometry, seed: int, expert: int, device="cpu"):
    """One local expert's (w13 fp8 [2I, H], s13 [2I/128, H/128], w2 fp8 [H, I], s2 [H/128, I/128])."""
    g = _gen(device, seed * 1000003 + 17 * expert + 5)
    w13 = torch.randn(2 * geo.inter, geo.hidden, generator=g, device=device) * 0.02
    q13, s13 = quantize_blocks_128(w13)
    del w13
    w2 = torch.randn(geo.hidden, geo.inter, generator=g, device=device) * 0.02
    q2, s2 = quantize_blocks_128(w2)
    return q13, s13, q2, s2


def make_weights(geo: Geometry, seed: int, device="cpu", experts=None):
    """All local experts' weights (or only ``experts``; the rest stay zero)."""
    E, I, H = geo.num_local, geo.inter, geo.hidden
    w13 = torch.zeros(E, 2 * I, H, dtype=torch.float8_e4m3fn, device=device)
    s13 = torch.ones(E, 2 * I // 128, H // 128, dtype=torch.float32, device=device)
    w2 = torch.zeros(E, H, I, dtype=torch.float8_e4m3fn, device=device)
    s2 = torch.ones(E, H // 128, I // 128, dtype=torch.float32, device=device)
    for e in range(E) if experts is None else experts:
        q13, a13, q2, a2 = make_expert(geo, seed, e, device)
        w13[e].copy_(q13)
        s13[e].copy_(a13)
        w2[e].copy_(q2)
        s2[e].copy_(a2)
    return dict(gemm1_weights=w13, gemm1_weights_scale=s13, gemm2_weights=w2,
                gemm2_weights_scale=s2)


def make_expert_slice(geo: Geometry, seed: int, first: int, count: int, device="cpu"):
    """Weights of global experts [first, first + count) (expert-parallel rank slice); the
    values are those `make_weights` gives the same experts, since each expert has its own
    generator keyed by (seed, expert id)."""
    return make_expert_set(geo, seed, range(first, first + count), device)


def make_expert_set(geo: Geometry, seed: int, experts, device="cpu"):
    """Weights of the global experts `experts`, stacked in that order (an expert-parallel
    rank's experts under any placement); each expert's values are those `make_weights`
    gives it."""
    experts = [int(e) for e in experts]
    count, I, H = len(experts), geo.inter, geo.hidden
    w13 = torch.empty(count, 2 * I, H, dtype=torch.float8_e4m3fn, device=device)
    s13 = torch.empty(count, 2 * I // 128, H // 128, dtype=torch.float32, device=device)
    w2 = torch.empty(count, H, I, dtype=torch.float8_e4m3fn, device=device)
    s2 = torch.empty(count, H // 128, I // 128, dtype=torch.float32, device=device)
    for j, e in enumerate(experts):
        q13, a13, q2, a2 = make_expert(geo, seed, e, device)
        w13[j].copy_(q13)
        s13[j].copy_(a13)
        w2[j].copy_(q2)
        s2[j].copy_(a2)
    return dict(gemm1_weights=w13, gemm1_weights_scale=s13, gemm2_weights=w2,
                gemm2_weights_scale=s2)


def make_inputs(geo: Geometry, T: int, seed: int, device="cpu", skew_hot: int = 0,
                local_expert_offset: int = 0, experts=None):
    acts = make_activations(geo, T, seed, device, skew_hot, local_expert_offset)
    ws = make_weights(geo, seed, device, experts)
    acts.update(ws)
    return acts


OPERATOR_ARGS = ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale",
                 "gemm1_weights", "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale")


def operator_args(inputs: dict):
    return [inputs[k] for k in OPERATOR_ARGS]
