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

Expert placement: by default rank r owns the contiguous experts [r*E/N, (r+1)*E/N), the
reference's slice (`local_expert_offset = r*E/N`). Routing skew makes those slices unequal
(with the DS-V3 config-3 workload the busiest of 8 slices has 1.3x the mean rows), and every
step waits for the busiest rank. `placement` assigns any E/N experts to each rank instead
(rank r owns placement[r*E/N : (r+1)*E/N], its weights stacked in that order).
`locality_placement` computes one from a calibration batch's routing that evens out the
ranks' work while keeping each token's experts on few ranks, `balanced_placement` one from
per-expert row counts alone; `calibrate_placement` routes the batch on every rank and
returns the same placement everywhere. Internally each routed expert id is replaced by its
position in the placement, so the destination rank is position // (E/N) and the local
operator runs with local_expert_offset = r*E/N, exactly as for the contiguous slices.

Without a host round trip (`max_tokens`): buffers are sized once, the counts are gathered
and the row offsets computed on the device, and the local operator reads the received token
count from device memory and returns its rows straight to the sources from its combine.

On CUDA the send plan, the payload packing and unpacking and the rank-ordered combine are
kernels of the library (`fmoe_ep_*` in include/fmoe.h: one launch each, instead of chains
of framework ops). With more than one rank the rows move over peer memory by default
(`exchange="p2p"`): every rank's receive and return buffers are mapped into the other
ranks by CUDA IPC, the pack kernel stores each payload row straight into its destination's
receive buffer over NVLink, and a return kernel stores each partial output row straight
into its source's return buffer; a one-element all-reduce on the stream orders the ranks
after each of the two kernels. Only the per-destination counts (and the token counts, for
sizing) are gathered to the host. `exchange="nccl"` moves the same rows with NCCL
all-to-all-v instead. The framework-op version below is the CPU restatement the gloo tests
exercise, and `fused_exchange=False` selects it on CUDA too.
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


def placement_cost(rows: torch.Tensor, tile_rows: int = 128) -> torch.Tensor:
    """Relative GEMM time of each expert: its routed rows in 128-row token tiles (every tile
    streams the expert's full weights through the tensor cores once)."""
    return (rows.to(torch.int64) + tile_rows - 1) // tile_rows


def balanced_placement(rows, world: int) -> list:
    """An expert placement for `world` ranks (E/world experts each) that evens out the
    ranks' GEMM work: experts by decreasing `placement_cost`, each to the rank with the
    least work so far that still has a free slot (longest-processing-time greedy; ties to
    the lower expert id and the lower rank, so every rank computes the same placement).
    Returns the E expert ids in rank-major order."""
    rows = torch.as_tensor(rows).to(torch.int64).cpu()
    E = rows.numel()
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    per = E // world
    cost = placement_cost(rows).tolist()
    order = sorted(range(E), key=lambda e: (-cost[e], e))
    work = [0] * world
    owned = [[] for _ in range(world)]
    for e in order:
        r = min((r for r in range(world) if len(owned[r]) < per), key=lambda r: (work[r], r))
        owned[r].append(e)
        work[r] += cost[e]
    return [e for r in range(world) for e in sorted(owned[r])]


# Relative cost of one token a rank receives, in 128-row GEMM tiles: a received token moves
# 7,456 B in and 14,336 B back over NVLink (≈ 0.031 ms per thousand at ≈ 700 GB/s), a tile
# of the 256-expert layer's GEMM1 + GEMM2 takes ≈ 4.25 µs on a B200 at ≈ 1,000 rows per
# expert (8-GPU expert parallelism).
RECV_TOKEN_COST_IN_TILES = 0.0073


def locality_placement(topk_idx, num_experts: int, world: int, max_swaps: int = 256,
                       recv_cost: float = RECV_TOKEN_COST_IN_TILES, search: str = "max-rank",
                       power: float = 16.0) -> list:
    """An expert placement that evens out the ranks' work while keeping each token's experts
    on few ranks. Starts from the contiguous slices (a DS-V3 routing group per rank at 8
    ranks, so a token goes to at most topk_group ranks) and swaps experts between ranks.
    Rank cost: cost(r) = tiles(r) + recv_cost * tokens_received(r), tiles counted as 128-row
    token tiles of each expert's routed rows and tokens_received the tokens of `topk_idx`
    ([T, K] expert ids of a calibration batch, all ranks' tokens) that need rank r.
    search "max-rank" (default): each step takes the swap of an expert of the most loaded
    rank that lowers the largest cost the most. search "pairs": each step takes the swap,
    over every pair of ranks, that lowers sum_r (cost(r) / mean cost) ** power the most (a
    smooth stand-in for the largest cost), and the placement with the lowest largest cost
    seen is returned; it balances the model cost better (8 ranks: busiest 1.034x the mean
    against 1.078x) but measured 1.2 % slower per step on 8 B200s (3.390 against 3.348 ms).
    Deterministic; returns the expert ids in rank-major order."""
    import numpy as np

    idx = torch.as_tensor(topk_idx).to(torch.int64).cpu().numpy()
    E = num_experts
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    if search not in ("pairs", "max-rank"):
        raise ValueError(f"unknown search {search!r}")
    per = E // world
    owner = np.arange(E) // per
    if world == 1 or idx.size == 0:
        return list(range(E))
    T = idx.shape[0]
    valid = (idx >= 0) & (idx < E)
    rows = np.bincount(idx[valid], minlength=E)
    tiles = (rows + 127) // 128
    X = np.zeros((E, T), dtype=bool)  # expert e is selected by token t
    for k in range(idx.shape[1]):
        m = valid[:, k]
        X[idx[m, k], np.nonzero(m)[0]] = True
    Xb = np.packbits(X, axis=1)
    C = np.zeros((world, T), dtype=np.int32)  # experts of token t on rank r
    for e in range(E):
        C[owner[e]] += X[e]
    load = np.array([tiles[owner == r].sum() for r in range(world)], dtype=np.float64)
    J = load + recv_cost * (C > 0).sum(1)
    scale = max(float(J.mean()), 1e-9)
    best_owner, best_max = owner.copy(), float(J.max())

    def swap_costs(a, b):
        # costs of ranks a and b after swapping expert ea[i] (on a) with fb[j] (on b)
        ea, fb = np.nonzero(owner == a)[0], np.nonzero(owner == b)[0]
        base_a = np.packbits(C[a] >= 2)[None, :] | (np.packbits(C[a] == 1)[None, :] & ~Xb[ea])
        base_b = np.packbits(C[b] >= 2)[None, :] | (np.packbits(C[b] == 1)[None, :] & ~Xb[fb])
        recv_a = np.bitwise_count(base_a[:, None, :] | Xb[fb][None, :, :]).sum(-1)
        recv_b = np.bitwise_count(base_b[None, :, :] | Xb[ea][:, None, :]).sum(-1)
        ja = load[a] - tiles[ea][:, None] + tiles[fb][None, :] + recv_cost * recv_a
        jb = load[b] + tiles[ea][:, None] - tiles[fb][None, :] + recv_cost * recv_b
        return ea, fb, ja, jb

    for _ in range(max_swaps):
        best = None
        if search == "pairs":
            for a in range(world):
                for b in range(a + 1, world):
                    ea, fb, ja, jb = swap_costs(a, b)
                    delta = ((ja / scale) ** power + (jb / scale) ** power
                             - (J[a] / scale) ** power - (J[b] / scale) ** power)
                    i, j = np.unravel_index(int(np.argmin(delta)), delta.shape)
                    if best is None or delta[i, j] < best[0]:
                        best = (float(delta[i, j]), int(ea[i]), int(fb[j]), a, b)
            if best is None or best[0] >= -1e-12:
                break
        else:
            a = int(np.argmax(J))
            rest = np.delete(J, a)
            for b in range(world):
                if b == a:
                    continue
                ea, fb, ja, jb = swap_costs(a, b)
                others = np.delete(rest, b - (b > a)).max() if world > 2 else -np.inf
                jn = np.maximum(np.maximum(ja, jb), others)
                i, j = np.unravel_index(int(np.argmin(jn)), jn.shape)
                if best is None or jn[i, j] < best[0]:
                    best = (float(jn[i, j]), int(ea[i]), int(fb[j]), a, b)
            if best is None or best[0] >= J.max() - 1e-9:
                break
        _, e, f, a, b = best
        owner[e], owner[f] = b, a
        C[a] += X[f].astype(np.int32) - X[e]
        C[b] += X[e].astype(np.int32) - X[f]
        load[a] += tiles[f] - tiles[e]
        load[b] += tiles[e] - tiles[f]
        J = load + recv_cost * (C > 0).sum(1)
        if J.max() < best_max - 1e-9:
            best_owner, best_max = owner.copy(), float(J.max())
    return [int(e) for r in range(world) for e in np.nonzero(best_owner == r)[0]]


def calibrate_placement(route_fn: RouteFn, routing_logits, routing_bias, num_experts: int,
                        group=None, mode: str = "balanced", search: str = "max-rank") -> list:
    """Route a calibration batch on every rank and return a placement computed from it, the
    same list on every rank: `balanced_placement` of the per-expert row counts added over
    the ranks (mode "balanced"), or `locality_placement` of every rank's routing (mode
    "local", the [T, K] ids all-gathered)."""
    idx, _ = route_fn(routing_logits, routing_bias)
    dist_on = dist.is_initialized() and dist.get_world_size(group) > 1
    world = dist.get_world_size(group) if dist_on else 1
    if mode == "local":
        ids = idx.to(torch.int32).contiguous()
        if dist_on:
            parts = [None] * world
            dist.all_gather_object(parts, ids.cpu(), group=group)
            ids = torch.cat(parts)
        return locality_placement(ids, num_experts, world, search=search)
    if mode != "balanced":
        raise ValueError(f"unknown placement mode {mode!r}")
    flat = idx.reshape(-1).long()
    rows = torch.bincount(flat[flat >= 0], minlength=num_experts).to(torch.int64)
    if dist_on:
        dist.all_reduce(rows, group=group)
    return balanced_placement(rows, world)


class ExpertParallelMoE:
    """The 256-expert layer sharded over the ranks of `group` by expert.

    `route_fn(logits, bias) -> (idx int32 [T, K], w fp32 [T, K])` and
    `local_fn(idx, w, hidden, scale, local_offset) -> bf16 [R, H]` default to the B200
    kernels of this package; tests pass CPU restatements to exercise the exchange logic.
    `placement` (E expert ids, rank-major; None = contiguous slices) decides which experts
    each rank owns; `weights` hold this rank's experts in `local_experts()` order, and
    `local_fn` sees expert ids replaced by their placement positions.
    """

    def __init__(self, num_experts: int = 256, n_group: int = 8, topk_group: int = 4,
                 top_k: int = 8, routed_scaling_factor: float = 2.5, group=None,
                 weights: Optional[dict] = None, route_fn: Optional[RouteFn] = None,
                 local_fn: Optional[LocalFn] = None, fused_exchange: bool = True,
                 exchange: str = "p2p", placement=None, max_tokens: Optional[int] = None,
                 fused_return: bool = True):
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
        if exchange not in ("p2p", "nccl"):
            raise ValueError(f"exchange must be 'p2p' or 'nccl', not {exchange!r}")
        self.exchange = exchange
        self.placement = None
        self._pos = None           # expert id -> placement position (None: identity)
        if placement is not None:
            pl = [int(e) for e in placement]
            if sorted(pl) != list(range(num_experts)):
                raise ValueError("placement must list every expert exactly once")
            if pl != list(range(num_experts)):
                self.placement = pl
                pos = [0] * num_experts
                for i, e in enumerate(pl):
                    pos[e] = i
                self._pos = torch.tensor(pos, dtype=torch.int32)
        if max_tokens is not None and max_tokens <= 0:
            raise ValueError("max_tokens must be positive")
        self.max_tokens = max_tokens
        self.fused_return = fused_return
        self._static = None      # device-side offset state of the host-sync-free P2P step
        self._peers = None       # fmoe_b200.PeerBuffers, sized for _cap_tokens per rank
        self._cap_tokens = 0
        self._flag = None
        self._err = None
        self._timed = False
        # filled by a timed forward on CUDA (see _local)
        self.local_stage_ms = None
        self.last_local_tokens = self.last_local_rows = self.last_local_active = 0

    def local_experts(self) -> list:
        """Global ids of the experts this rank owns, in the order its weights are stacked."""
        lo = self.local_offset
        if self.placement is None:
            return list(range(lo, lo + self.e_per_rank))
        return self.placement[lo:lo + self.e_per_rank]

    def place_ids(self, idx: torch.Tensor) -> torch.Tensor:
        """Expert ids -> placement positions (unselected slots, < 0, stay as they are)."""
        if self._pos is None:
            return idx
        if self._pos.device != idx.device:
            self._pos = self._pos.to(idx.device)
        return torch.where(idx >= 0, self._pos[idx.clamp_min(0).long()], idx)

    def _dev_pos(self, dev):
        """The placement positions on `dev` (None for contiguous slices)."""
        if self._pos is not None and self._pos.device != dev:
            self._pos = self._pos.to(dev)
        return self._pos

    # ---- default B200 implementations --------------------------------------------------
    def _route_gpu(self, logits, bias):
        import fmoe_b200

        # only the (id, weight) pairs are used here: the routing kernel's local plan is kept
        # to one expert (the receiving ranks plan their own experts)
        return fmoe_b200.route(logits, bias, self.n_group, self.topk_group, self.top_k,
                               self.rsf, num_local_experts=1, local_expert_offset=0)

    def _local_gpu(self, idx, w, hs, sc, offset, count=None, out=None, return_to=None):
        import fmoe_b200

        ws = self.weights
        return fmoe_b200.forward_routed(idx, w, hs, sc, ws["gemm1_weights"],
                                        ws["gemm1_weights_scale"], ws["gemm2_weights"],
                                        ws["gemm2_weights_scale"], offset, self.num_experts,
                                        n_group=self.n_group, topk_group=self.topk_group,
                                        num_tokens_dev=count, out=out, return_to=return_to)

    # ---- peer-memory exchange -----------------------------------------------------------
    def _barrier(self):
        # stream-ordered: the next kernels of every rank wait for every rank's previous ones
        dist.all_reduce(self._flag, group=self.group)

    def _ensure_peers(self, t_max: int, H: int, K: int, dev):
        """(Re)allocate the IPC-shared buffers for t_max tokens per rank. Every rank calls
        this with the same t_max (gathered), so the collective steps match."""
        import fmoe_b200

        if self._peers is not None and t_max <= self._cap_tokens:
            return
        if self._peers is not None:
            self._barrier()
            torch.cuda.synchronize(dev)
            self._peers.close()
        cap = max(64, 1 << (max(t_max, 1) - 1).bit_length())
        rows = cap * self.world  # a token goes to each rank at most once
        self._peers = fmoe_b200.PeerBuffers(rows * fmoe_b200.ep_payload_bytes(H, K),
                                            rows * H * 2, self.group, dev)
        self._cap_tokens = cap
        if self._flag is None:
            self._flag = torch.zeros(1, dtype=torch.int32, device=dev)
            self._err = torch.zeros(1, dtype=torch.int32, device=dev)

    def exchange_error(self) -> int:
        """Bits set by the P2P kernels since the last forward (0 = every row in bounds)."""
        return int(self._err.item()) if self._err is not None else 0

    def close(self):
        if self._peers is not None:
            self._barrier()
            torch.cuda.synchronize()
            self._peers.close()
            self._peers = None
            self._static = None

    def _forward_p2p(self, idx, w, hidden_states, hidden_states_scale, mark):
        import fmoe_b200

        T, H = hidden_states.shape
        K, world, me = self.top_k, self.world, self.rank
        dev = hidden_states.device
        pos, _, counts = fmoe_b200.ep_plan(idx, world, self.e_per_rank, self._dev_pos(dev))
        meta = torch.cat([counts.to(torch.int64),
                          torch.tensor([T], dtype=torch.int64, device=dev)])
        allm = torch.empty(world, world + 1, dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(allm, meta, group=self.group)
        m = allm.tolist()
        cnt = [row[:world] for row in m]  # cnt[s][d]: rows rank s sends to rank d
        self._ensure_peers(max(row[world] for row in m), H, K, dev)
        cap = self._cap_tokens * world

        def src_start(d, s):  # first row of source s in rank d's receive buffer
            return sum(cnt[q][d] for q in range(s))

        def seg_base(s, d):  # first row of destination d in rank s's send order
            return sum(cnt[s][:d])

        shift_pack = [src_start(d, me) - seg_base(me, d) for d in range(world)]
        starts = [src_start(me, s) for s in range(world + 1)]
        shift_ret = [seg_base(s, me) - starts[s] for s in range(world)]
        R = starts[world]
        # the three offset tables in one pinned, asynchronous upload
        host = torch.tensor(shift_pack + starts + shift_ret, dtype=torch.int64).pin_memory()
        tables = torch.empty(host.numel(), dtype=torch.int64, device=dev)
        tables.copy_(host, non_blocking=True)
        shift_pack_t = tables[:world]
        starts_t = tables[world:2 * world + 1]
        shift_ret_t = tables[2 * world + 1:]
        self._err.zero_()
        fmoe_b200.ep_pack_p2p(hidden_states, hidden_states_scale, idx, w, pos, self._peers,
                              shift_pack_t, cap, self._err)
        self._barrier()
        hs_r, sc_r, idx_r, w_r = fmoe_b200.ep_unpack(self._peers.recv[me], H, K, rows=R,
                                                     device=dev)
        mark()
        part = self._local(idx_r, w_r, hs_r, sc_r)
        mark()
        fmoe_b200.ep_return_p2p(part.contiguous(), starts_t, self._peers, shift_ret_t, cap,
                                self._err)
        self._barrier()
        return fmoe_b200.ep_combine(self._peers.back[me], pos, T, H)

    def _forward_p2p_static(self, idx, w, hidden_states, hidden_states_scale, mark):
        """The P2P step without a host round trip (`max_tokens` set): buffers sized once for
        max_tokens per rank; the per-destination counts are all-gathered on the device, the
        row offsets and the received row count computed there (fmoe_ep_offsets), and the
        unpack and the local operator take that count from device memory, so the host only
        enqueues work and the local operator replays one cached graph. The operator's
        combine writes the partial rows straight into the sources' return buffers
        (fmoe_forward_routed_count_p2p), so no separate return pass runs."""
        import fmoe_b200

        T, H = hidden_states.shape
        K, world, me = self.top_k, self.world, self.rank
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens={self.max_tokens}")
        dev = hidden_states.device
        if self._static is None:
            self._ensure_peers(self.max_tokens, H, K, dev)  # collective, same size on every rank
            cap = self._cap_tokens * world
            self._static = {
                "cap": cap,
                "meta": torch.zeros(world + 1, dtype=torch.int64, device=dev),
                "allm": torch.empty(world, world + 1, dtype=torch.int64, device=dev),
                "tables": torch.empty(3 * world + 1, dtype=torch.int64, device=dev),
                "rows": torch.zeros(1, dtype=torch.int32, device=dev),
                "unpacked": (torch.empty(cap, H, dtype=torch.float8_e4m3fn, device=dev),
                             torch.empty(H // 128, cap, dtype=torch.float32, device=dev),
                             torch.empty(cap, K, dtype=torch.int32, device=dev),
                             torch.empty(cap, K, dtype=torch.float32, device=dev)),
                "part": torch.empty(cap, H, dtype=torch.bfloat16, device=dev),
            }
        st = self._static
        cap = st["cap"]
        pos, _, counts = fmoe_b200.ep_plan(idx, world, self.e_per_rank, self._dev_pos(dev))
        st["meta"][:world].copy_(counts)
        dist.all_gather_into_tensor(st["allm"], st["meta"], group=self.group)
        tables, rows = fmoe_b200.ep_offsets(st["allm"], me, st["tables"], st["rows"])
        self._err.zero_()
        fmoe_b200.ep_pack_p2p(hidden_states, hidden_states_scale, idx, w, pos, self._peers,
                              tables[:world], cap, self._err)
        self._barrier()
        hs_r, sc_r, idx_r, w_r = fmoe_b200.ep_unpack_count(self._peers.recv[me], cap, rows, H, K,
                                                           out=st["unpacked"], device=dev)
        mark()
        if self.fused_return:
            # the operator's combine stores each partial row straight into its source's buffer
            self._local(idx_r, w_r, hs_r, sc_r, count=rows, out=st["part"],
                        return_to=(self._peers, tables[world:2 * world + 1],
                                   tables[2 * world + 1:], cap, self._err))
            mark()
        else:
            part = self._local(idx_r, w_r, hs_r, sc_r, count=rows, out=st["part"])
            mark()
            fmoe_b200.ep_return_p2p(part, tables[world:2 * world + 1], self._peers,
                                    tables[2 * world + 1:], cap, self._err)
        self._barrier()
        return fmoe_b200.ep_combine(self._peers.back[me], pos, T, H)

    def _local(self, idx_r, w_r, hs_r, sc_r, count=None, out=None, return_to=None):
        """The rank's own experts on what it received (`count`: device token count, the
        tensors then sized for a capacity). In a timed pass on CUDA with the default
        kernels, also records the operator's stage times (route, permute, gemm1, gemm2,
        combine) and the received tokens, routed rows and active experts."""
        if count is not None:
            if self.local_fn != self._local_gpu:
                raise ValueError("a device-side token count needs the default local operator")
            run = lambda: self._local_gpu(idx_r, w_r, hs_r, sc_r, self.local_offset,  # noqa
                                          count=count, out=out, return_to=return_to)
        else:
            run = lambda: self.local_fn(idx_r, w_r, hs_r, sc_r, self.local_offset)  # noqa
        if not (self._timed and hs_r.device.type == "cuda" and self.local_fn == self._local_gpu):
            return run()
        import fmoe_b200

        n = int(count.item()) if count is not None else int(idx_r.shape[0])
        lo, hi = self.local_offset, self.local_offset + self.e_per_rank
        ids = idx_r[:n]
        sel = ids[(ids >= lo) & (ids < hi)]
        self.last_local_tokens = n
        self.last_local_rows = int(sel.numel())
        self.last_local_active = int(torch.unique(sel).numel())
        st = fmoe_b200.StageTimer()
        with st:
            part = run()
        torch.cuda.synchronize()
        self.local_stage_ms = st.times_ms()
        return part

    # ---- the layer -------------------------------------------------------------------------
    def forward(self, routing_logits, routing_bias, hidden_states, hidden_states_scale,
                timed: bool = False) -> torch.Tensor:
        T, H = hidden_states.shape
        K = self.top_k
        dev = hidden_states.device
        ev = []
        self._timed = timed

        def mark():
            if timed and dev.type == "cuda":
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                ev.append(e)

        mark()
        idx, w = self.route_fn(routing_logits, routing_bias)
        idx = idx.to(torch.int32).contiguous()
        w = w.to(torch.float32).contiguous()
        fused = self.fused_exchange and dev.type == "cuda"
        if not fused:
            idx = self.place_ids(idx)  # (fused: fmoe_ep_plan_placed maps the ids in place)
        mark()
        if fused and self.world > 1 and self.exchange == "p2p":
            step = self._forward_p2p_static if self.max_tokens else self._forward_p2p
            res = step(idx, w, hidden_states, hidden_states_scale, mark)
            mark()
            if timed and len(ev) == 5:
                torch.cuda.synchronize()
                self.timings = EPTimings(ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]),
                                         ev[2].elapsed_time(ev[3]), ev[3].elapsed_time(ev[4]))
            return res
        if fused:
            import fmoe_b200

            pos, _, counts = fmoe_b200.ep_plan(idx, self.world, self.e_per_rank,
                                               self._dev_pos(dev))
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
        part = self._local(idx_r, w_r, hs_r, sc_r)
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
