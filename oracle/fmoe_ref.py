"""CPU oracle for the fused FP8 block-scaled DeepSeek-V3 MoE operator.

TEST INFRASTRUCTURE ONLY: the checker for the CUDA path. Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import this
module. The product library never imports it.

Two parts:

* ``route`` / ``plan`` call the C restatement in ``fmoe_oracle.c`` (built to
  ``oracle/liboracle.so``). They must agree with the CUDA kernels bit for bit.
* ``moe_forward`` is the dequantise-to-fp32 PyTorch CPU restatement of the operator
  definition, following the reference ``solution/cuda/kernel.cu``:

  - activation dequant ``A[r, c] = fp8(hs[t, c]) * hs_scale[c // 128, t]``  (kernel.cu:781-782)
  - weight dequant ``W[n, c] = fp8(w[e, n, c]) * w_scale[e, n // 128, c // 128]`` (kernel.cu:919-921)
  - ``G1 = A @ W13^T``; ``C = G1[:, :I] * silu(G1[:, I:])``  (kernel.cu:818-832)
  - ``O = C @ W2^T``  (kernel.cu:1104-1199)
  - ``out[t] = sum over local routes of w[t, k] * O[row]``, local means
    ``0 <= idx - local_expert_offset < E_local``  (kernel.cu:835-891)
  - output cast to bf16  (kernel.cu:519-528)

  It runs in fp32 on the host cores. ``torch.set_num_threads`` controls the core
  count, which the caller reports.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np
import torch

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle.so"
_lib = None


def build(force: bool = False) -> Path:
    """Compile fmoe_oracle.c into oracle/liboracle.so (no fast-math, no FMA contraction)."""
    src = _HERE / "fmoe_oracle.c"
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.check_call(
            ["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
             str(src), "-o", str(_LIB_PATH), "-lm"])
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        lib.fmoe_oracle_route.restype = ctypes.c_int
        lib.fmoe_oracle_route.argtypes = [
            ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_void_p]
        lib.fmoe_oracle_plan.restype = ctypes.c_int64
        lib.fmoe_oracle_plan.argtypes = [
            ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_int64]
        lib.fmoe_oracle_sigmoid.restype = ctypes.c_float
        lib.fmoe_oracle_sigmoid.argtypes = [ctypes.c_float]
        lib.fmoe_oracle_expf.restype = ctypes.c_float
        lib.fmoe_oracle_expf.argtypes = [ctypes.c_float]
        _lib = lib
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def sigmoid(x: np.ndarray) -> np.ndarray:
    lib = _load()
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    return np.array([lib.fmoe_oracle_sigmoid(float(v)) for v in x], dtype=np.float32)


def route(logits, bias, n_group: int, topk_group: int, top_k: int, rsf: float,
          return_scores: bool = False):
    """Bit-exact routing restatement (kernel.cu:388-516).

    logits: fp32 [T, E] (torch or numpy); bias: bf16 [E] torch tensor or uint16 bits.
    Returns (idx int32 [T, K], w fp32 [T, K]) numpy arrays (+ sigmoid scores).
    """
    lib = _load()
    lg = np.ascontiguousarray(_np(logits), dtype=np.float32)
    T, E = lg.shape
    b = _bf16_bits(bias)
    idx = np.empty((T, top_k), dtype=np.int32)
    w = np.empty((T, top_k), dtype=np.float32)
    s = np.empty((T, E), dtype=np.float32) if return_scores else None
    rc = lib.fmoe_oracle_route(T, E, n_group, topk_group, top_k, _ptr(lg), _ptr(b),
                               float(rsf), _ptr(idx), _ptr(w),
                               _ptr(s) if s is not None else None)
    if rc != 0:
        raise ValueError("oracle route: unsupported geometry")
    return (idx, w, s) if return_scores else (idx, w)


def plan(topk_idx: np.ndarray, E_local: int, local_offset: int, row_cap: int):
    """Deterministic expert-major row plan (kernel.cu:530-592, stable order)."""
    lib = _load()
    ti = np.ascontiguousarray(topk_idx, dtype=np.int32)
    T, K = ti.shape
    cnt = np.zeros(E_local, np.int32)
    off = np.zeros(E_local + 1, np.int32)
    row_token = np.empty(row_cap, np.int32)
    row_k = np.empty(row_cap, np.int32)
    token_row = np.empty((T, K), np.int32)
    total = lib.fmoe_oracle_plan(T, K, E_local, local_offset, _ptr(ti), _ptr(cnt), _ptr(off),
                                 _ptr(row_token), _ptr(row_k), _ptr(token_row), row_cap)
    if total < 0:
        raise ValueError("oracle plan: row_cap too small")
    return dict(expert_cnt=cnt, expert_off=off, row_token=row_token, row_k=row_k,
                token_row=token_row, total=int(total))


def _np(x):
    if isinstance(x, torch.Tensor):
        return x.detach().cpu().numpy()
    return np.asarray(x)


def _bf16_bits(bias) -> np.ndarray:
    if isinstance(bias, torch.Tensor):
        assert bias.dtype == torch.bfloat16
        return np.ascontiguousarray(bias.detach().cpu().view(torch.int16).numpy().view(np.uint16))
    return np.ascontiguousarray(np.asarray(bias, dtype=np.uint16))


def route_definition(logits: torch.Tensor, bias: torch.Tensor, n_group: int, topk_group: int,
                     top_k: int, rsf: float):
    """Routing written the way a PyTorch definition would (torch.sigmoid, torch.topk).

    Used only to report how often the exact sigmoid and torch's sigmoid disagree on
    the selected set (near ties); it is not the parity oracle.
    """
    lg = logits.float().cpu()
    s = torch.sigmoid(lg)
    swb = s + bias.float().cpu()
    T, E = lg.shape
    G = E // n_group
    grp = swb.view(T, n_group, G).topk(2, dim=-1).values.sum(-1)
    gidx = grp.topk(topk_group, dim=-1, sorted=False).indices
    mask = torch.zeros(T, n_group, dtype=torch.bool).scatter_(1, gidx, True)
    emask = mask.unsqueeze(-1).expand(T, n_group, G).reshape(T, E)
    cand = swb.masked_fill(~emask, float("-inf"))
    idx = cand.topk(top_k, dim=-1).indices
    ws = s.gather(1, idx)
    w = ws / (ws.sum(-1, keepdim=True) + 1e-20) * rsf
    return idx.to(torch.int32).numpy(), w.numpy()


def dequant_act(hs_fp8: torch.Tensor, hs_scale: torch.Tensor, rows=None) -> torch.Tensor:
    """A = fp8(hs) * scale[c // 128, t]  (kernel.cu:781-782). hs_scale is [H/128, T]."""
    hs = hs_fp8.cpu()
    sc = hs_scale.cpu().float()
    if rows is not None:
        hs = hs[rows]
        sc = sc[:, rows]
    a = hs.float()
    return a * sc.t().repeat_interleave(128, dim=1)


def dequant_weight(w_fp8: torch.Tensor, w_scale: torch.Tensor) -> torch.Tensor:
    """W = fp8(w) * scale[n // 128, c // 128]  (kernel.cu:919-921), one expert."""
    w = w_fp8.cpu().float()
    s = w_scale.cpu().float().repeat_interleave(128, 0).repeat_interleave(128, 1)
    return w * s


def moe_forward(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                local_expert_offset: int, routed_scaling_factor: float,
                n_group: int, topk_group: int, top_k: int, return_aux: bool = False,
                weight_cache: dict | None = None):
    """Dequantise-to-fp32 CPU reference of the whole operator; returns bf16 [T, H].

    The weight tensors may live on any device; only experts that receive rows are
    dequantised, one at a time, so the DS-V3 shapes fit in host memory. A dict passed
    as ``weight_cache`` keeps the dequantised experts between calls on the same weights.
    """
    idx, w = route(routing_logits, routing_bias, n_group, topk_group, top_k,
                   routed_scaling_factor)
    out = moe_forward_routed(idx, w, hidden_states, hidden_states_scale, gemm1_weights,
                             gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                             local_expert_offset, weight_cache=weight_cache, fp32=True)
    res = out.to(torch.bfloat16)
    if return_aux:
        return res, dict(topk_idx=idx, topk_w=w, out_f32=out)
    return res


def moe_forward_routed(topk_idx, topk_w, hidden_states, hidden_states_scale, gemm1_weights,
                       gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                       local_expert_offset: int, weight_cache: dict | None = None,
                       fp32: bool = False):
    """The operator after routing: out[t] = sum over (t, k) with a local expert of
    w[t, k] * GEMM2(SwiGLU(GEMM1(A_t))) (kernel.cu:761-891), fp32 on the host cores.
    Returns fp32 [T, H] when ``fp32`` else bf16."""
    idx = _np(topk_idx).astype(np.int32)
    w = _np(topk_w).astype(np.float32)
    T = idx.shape[0]
    E_local, two_i, H = gemm1_weights.shape
    I = two_i // 2
    out = torch.zeros(T, H, dtype=torch.float32)
    w_t = torch.from_numpy(w)
    for le in range(E_local):
        ge = le + local_expert_offset
        tok, kk = np.nonzero(idx == ge)
        if tok.size == 0:
            continue
        order = np.lexsort((kk, tok))
        tok, kk = tok[order], kk[order]
        a = dequant_act(hidden_states, hidden_states_scale, rows=torch.from_numpy(tok))
        if weight_cache is not None and le in weight_cache:
            w13, w2 = weight_cache[le]
        else:
            w13 = dequant_weight(gemm1_weights[le], gemm1_weights_scale[le])
            w2 = dequant_weight(gemm2_weights[le], gemm2_weights_scale[le])
            if weight_cache is not None:
                weight_cache[le] = (w13, w2)
        g1 = a @ w13.t()
        x1, x2 = g1[:, :I], g1[:, I:]
        c = x1 * (x2 / (1.0 + torch.exp(-x2)))
        o = c @ w2.t()
        wt = w_t[torch.from_numpy(tok), torch.from_numpy(kk)].unsqueeze(1)
        out.index_add_(0, torch.from_numpy(tok), o * wt)
    return out if fp32 else out.to(torch.bfloat16)


def route_margin(logits, bias, n_group, topk_group, top_k) -> float:
    """Smallest gap between the K-th selected and the best unselected biased score."""
    idx, _, s = route(logits, bias, n_group, topk_group, top_k, 1.0, return_scores=True)
    swb = s + _np(bias.float() if isinstance(bias, torch.Tensor) else bias).astype(np.float32)
    margin = np.inf
    for t in range(idx.shape[0]):
        sel = set(int(i) for i in idx[t] if i >= 0)
        kth = min(swb[t, i] for i in sel)
        rest = [swb[t, e] for e in range(swb.shape[1]) if e not in sel]
        if rest:
            margin = min(margin, float(kth - max(rest)))
    return margin
