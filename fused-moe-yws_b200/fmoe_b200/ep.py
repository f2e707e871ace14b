"""Expert-parallel fused MoE layer: the full 256-expert DeepSeek-V3 layer over N ranks.

The reference operator computes one 32-expert slice per call (`local_expert_offset`,
solution/cuda/kernel.cu:540-544, :572-586, :857-859) and leaves the exchange of tokens and
partial outputs between GPUs to its caller. This module is that caller, one process per
GPU over `torch.distributed` (NCCL on B200s, gloo for the CPU tests):

1. each rank routes its own tokens once (routing kernel, exact sigmoid);
2. a token goes to every rank that owns at least one of its top-k experts (rank r owns
   experts [r*E/N, (r+1)*E/N)); with DS-V3 group-limited routing that is at most
   topk_group ranks at N = 8, where rank r owns exactly routing group r;
3. counts are exchanged (all-to-all of N int64), then one all-to-all-v moves each token's
   FP8 row, its 128-block scales and its (expert id, weight) pairs;
4. each rank runs the fused operator on what it received, with the routing it was given
   (`fmoe_forward_routed`), producing per-token sums over its own experts;
5. a second all-to-all-v returns those partial outputs (bf16) to the token's rank, which
   adds them in rank order (deterministic) and casts to bf16.

The token order inside every message is ascending token id, so dispatch, compute and
combine are all deterministic.

On CUDA the send plan, the payload packing and unpacking and the rank-ordered combine are
kernels of the library (`fmoe_ep_*` in include/fmoe.h: one launch each, instead of chains
of framework ops); only the counts cross to the host, because NCCL's all-to-all-v takes
its split sizes there. The framework-op version below is the CPU restatement the gloo
tests exercise, and `fused_exchange=False` selects it on CUDA too.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist

RouteFn = Callable[[torch.Tensor, torch.Tensor], tuple]
LocalFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, int], torch.Tensor]


@dataclass
class EPTimings:
    """Host-side breakdown of the last forward (filled when `timed=True`)."""
    route_ms: float = 0.0
    dispatch_ms: float = 0.0
    compute_ms: float = 0.0
    combine_ms: float = 0.0


def pack_rows(hidden_states, hidden_states_scale, topk_idx, topk_w, tokens):
    """Per-token payload rows (uint8): FP8 row | block scales | expert ids | weights."""
    hs = hidden_states.view(torch.uint8)[tokens]
    sc = hidden_states_scale.t()[tokens].contiguous().view(torch.uint8)
    ii = topk_idx[tokens].contiguous().view(torch.uint8)
    ww = topk_w[tokens].contiguous().view(torch.uint8)
    return torch.cat([hs, sc, ii, ww], dim=1)


def unpack_rows(buf, H, K):
    """Inverse of pack_rows: (hidden fp8 [R, H], scale fp32 [H/128, R], idx, w)."""
    kb = H // 128
    hs = buf[:, :H].contiguous().view(torch.float8_e4m3fn)
    sc = buf[:, H:H + 4 * kb].contiguous().view(torch.float32).t().contiguous()
    ii = buf[:, H + 4 * kb:H + 4 * kb + 4 * K].contiguous().view(torch.int32)
    ww = buf[:, H + 4 * kb + 4 * K:].contiguous().view(torch.float32)
    return hs, sc, ii, ww


class ExpertParallelMoE:
    """The 256-expert layer sharded over the ranks of `group` by expert.

    `route_fn(logits, bias) -> (idx int32 [T, K], w fp32 [T, K])` and
    `local_fn(idx, w, hidden, scale, local_offset) -> bf16 [R, H]` default to the B200
    kernels of this package; tests pass CPU restatements to exercise the exchange logic.
    """

    def __init__(self, num_experts: int = 256, n_group: int = 8, topk_group: int = 4,
                 top_k: int = 8, routed_scaling_factor: float = 2.5, group=None,
                 weights: Optional[dict] = None, route_fn: Optional[RouteFn] = None,
                 local_fn: Optional[LocalFn] = None, fused_exchange: bool = True):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split over {self.world} ranks")
        self.num_experts = num_experts
        self.e_per_rank = num_experts // self.world
        self.local_offset = self.rank * self.e_per_rank
        self.n_group, self.topk_group, self.top_k = n_group, topk_group, top_k
        self.rsf = routed_scaling_factor
        self.weights = weights
        self.route_fn = route_fn or self._route_gpu
        self.local_fn = local_fn or self._local_gpu
        self.timings = EPTimings()
        self.fused_exchange = fused_exchange

    # ---- default B200 implementations --------------------------------------------------
    def _route_gpu(self, logits, bias):
        import fmoe_b200

        return fmoe_b200.route(logits, bias, self.n_group, self.topk_group, self.top_k,
                               self.rsf, num_local_experts=self.e_per_rank,
                               local_expert_offset=self.local_offset)

    def _local_gpu(self, idx, w, hs, sc, offset):
        import fmoe_b200

        ws = self.weights
        return fmoe_b200.forward_routed(idx, w, hs, sc, ws["gemm1_weights"],
                                        ws["gemm1_weights_scale"], ws["gemm2_weights"],
                                        ws["gemm2_weights_scale"], offset, self.num_experts,
                                        n_group=self.n_group, topk_group=self.topk_group)

    # ---- the layer -------------------------------------------------------------------------
    def forward(self, routing_logits, routing_bias, hidden_states, hidden_states_scale,
                timed: bool = False) -> torch.Tensor:
        T, H = hidden_states.shape
        K = self.top_k
        dev = hidden_states.device
        ev = []

        def mark():
            if timed and dev.type == "cuda":
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                ev.append(e)

        mark()
        idx, w = self.route_fn(routing_logits, routing_bias)
        idx = idx.to(torch.int32).contiguous()
        w = w.to(torch.float32).contiguous()
        mark()
        fused = self.fused_exchange and dev.type == "cuda"
        if fused:
            import fmoe_b200

            pos, _, counts = fmoe_b200.ep_plan(idx, self.world, self.e_per_rank)
            send_counts = counts.to(torch.int64)
        else:
            # destinations: rank owning each selected expert (unselected slots are -1)
            owner = torch.where(idx >= 0, idx // self.e_per_rank, torch.full_like(idx, -1))
            mask = torch.zeros(T, self.world, dtype=torch.bool, device=dev)
            valid = owner >= 0
            rows = torch.arange(T, device=dev).unsqueeze(1).expand(T, K)
            mask[rows[valid], owner[valid].long()] = True
            send_counts = mask.sum(0).to(torch.int64)
            order = torch.nonzero(mask.t(), as_tuple=False)  # (dest, token), by dest, token
            tokens = order[:, 1]
        recv_counts = torch.empty_like(send_counts)
        if self.world > 1:
            dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        else:
            recv_counts.copy_(send_counts)
        send_splits = send_counts.tolist()
        recv_splits = recv_counts.tolist()
        if fused:
            payload = fmoe_b200.ep_pack(hidden_states, hidden_states_scale, idx, w, pos,
                                        sum(send_splits))
        else:
            payload = pack_rows(hidden_states, hidden_states_scale, idx, w, tokens)
        recv = torch.empty(sum(recv_splits), payload.shape[1], dtype=torch.uint8, device=dev)
        if self.world > 1:
            dist.all_to_all_single(recv, payload, recv_splits, send_splits, group=self.group)
        else:
            recv.copy_(payload)
        if fused:
            hs_r, sc_r, idx_r, w_r = fmoe_b200.ep_unpack(recv, H, K)
        else:
            hs_r, sc_r, idx_r, w_r = unpack_rows(recv, H, K)
        mark()
        part = self.local_fn(idx_r, w_r, hs_r, sc_r, self.local_offset)
        mark()
        back = torch.empty(sum(send_splits), H, dtype=torch.bfloat16, device=dev)
        if self.world > 1:
            dist.all_to_all_single(back, part.contiguous(), send_splits, recv_splits,
                                   group=self.group)
        else:
            back.copy_(part)
        if fused:
            res = fmoe_b200.ep_combine(back, pos, T)
        else:
            out = torch.zeros(T, H, dtype=torch.float32, device=dev)
            start = 0
            for n in send_splits:  # rank order: each token's partials are added in order
                if n:
                    out.index_add_(0, tokens[start:start + n], back[start:start + n].float())
                start += n
            res = out.to(torch.bfloat16)
        mark()
        if timed and len(ev) == 5:
            torch.cuda.synchronize()
            self.timings = EPTimings(ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]),
                                     ev[2].elapsed_time(ev[3]), ev[3].elapsed_time(ev[4]))
        return res
