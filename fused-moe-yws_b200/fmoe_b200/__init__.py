"""B200-native fused FP8 block-scaled DeepSeek-V3 MoE operator (Python host mirror).

``kernel(...)`` has the argument order, tensor contract and error behaviour of the
reference operator (YuWei-CH/Fused-MoE-YWS ``solution/cuda/kernel.cu:1727-1837``, and its
Python global ``flashinfer.kernel`` in ``solution/cuda/binding.py:49-73``):

* ``ValueError`` for a wrong device, layout, rank or shape (``kernel.cu:121-168``);
* ``TypeError`` for a wrong dtype (``kernel.cu:145-150``);
* ``RuntimeError`` for CUDA failures (``kernel.cu:53-62``).

All work happens in ``lib/libfmoe.so`` (hand-written sm_100a CUDA behind the C ABI in
``include/fmoe.h``). There is no fallback: if the library or a CUDA device is missing,
calls raise ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

from . import workloads  # noqa: F401  (seeded synthetic inputs)
from .workloads import ROUTING_BY_EXPERTS

_PKG_ROOT = Path(__file__).resolve().parent.parent
LIB_PATH = _PKG_ROOT / "lib" / "libfmoe.so"
TVM_FFI_LIB_PATH = _PKG_ROOT / "lib" / "libfmoe_tvm_ffi.so"

FMOE_OK, FMOE_ERR_VALUE, FMOE_ERR_TYPE, FMOE_ERR_RUNTIME, FMOE_ERR_WORKSPACE, FMOE_ERR_DEVICE = range(6)

EXPORTED_SYMBOLS = ("fmoe_abi_version", "fmoe_last_error", "fmoe_validate", "fmoe_workspace_size",
                    "fmoe_autotune_tile_n", "fmoe_forward", "fmoe_route", "fmoe_read_device_error",
                    "fmoe_plan_view_get", "fmoe_set_stage_events", "fmoe_route_static",
                    "fmoe_forward_routed", "fmoe_selftest_wait_timeout", "fmoe_ep_plan",
                    "fmoe_ep_pack", "fmoe_ep_unpack", "fmoe_ep_combine", "fmoe_ep_ipc_alloc",
                    "fmoe_ep_ipc_open", "fmoe_ep_ipc_close", "fmoe_ep_ipc_free",
                    "fmoe_ep_pack_p2p", "fmoe_ep_return_p2p", "fmoe_poll_device_error",
                    "fmoe_selftest_inject_device_error", "fmoe_probe_fp8_mma_rate",
                    "fmoe_tile_n", "fmoe_prelayout_weights", "fmoe_forward_prelaid",
                    "fmoe_ep_plan_placed", "fmoe_forward_routed_count", "fmoe_ep_unpack_count",
                    "fmoe_ep_offsets", "fmoe_forward_routed_count_p2p",
                    "fmoe_forward_routed_prelaid")


class FmoeProblem(ctypes.Structure):
    _fields_ = [("num_tokens", ctypes.c_int64), ("num_experts", ctypes.c_int32),
                ("num_local_experts", ctypes.c_int32), ("hidden_size", ctypes.c_int32),
                ("intermediate_size", ctypes.c_int32), ("top_k", ctypes.c_int32),
                ("n_group", ctypes.c_int32), ("topk_group", ctypes.c_int32),
                ("local_expert_offset", ctypes.c_int32), ("routed_scaling_factor", ctypes.c_float),
                ("tile_n", ctypes.c_int32)]


class FmoeTensors(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "routing_logits", "routing_bias", "hidden_states", "hidden_states_scale", "gemm1_weights",
        "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale", "output")]


class FmoeRouteOut(ctypes.Structure):
    _fields_ = [("topk_idx", ctypes.c_void_p), ("topk_w", ctypes.c_void_p)]


class FmoePlanView(ctypes.Structure):
    _fields_ = [("expert_cnt", ctypes.c_void_p), ("expert_off", ctypes.c_void_p),
                ("row_token", ctypes.c_void_p), ("token_row", ctypes.c_void_p),
                ("meta", ctypes.c_void_p), ("row_cap", ctypes.c_int64)]


_lib = None
_lib_lock = threading.Lock()


def load_library(path: Path | str | None = None):
    """Load (once) and return the ctypes handle of libfmoe.so; raises if it is missing."""
    global _lib
    with _lib_lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"fused MoE library not built: {p} (run `python fused-moe-yws_b200/build.py`)")
        lib = ctypes.CDLL(str(p))
        lib.fmoe_abi_version.restype = ctypes.c_int
        lib.fmoe_last_error.restype = ctypes.c_char_p
        lib.fmoe_validate.argtypes = [ctypes.POINTER(FmoeProblem)]
        lib.fmoe_workspace_size.argtypes = [ctypes.POINTER(FmoeProblem),
                                            ctypes.POINTER(ctypes.c_size_t)]
        lib.fmoe_autotune_tile_n.argtypes = [ctypes.c_int64]
        lib.fmoe_tile_n.argtypes = [ctypes.POINTER(FmoeProblem)]
        lib.fmoe_prelayout_weights.argtypes = [ctypes.POINTER(FmoeProblem), ctypes.c_void_p,
                                               ctypes.c_void_p, ctypes.c_void_p,
                                               ctypes.c_void_p, ctypes.c_void_p]
        lib.fmoe_forward.argtypes = [ctypes.POINTER(FmoeProblem), ctypes.POINTER(FmoeTensors),
                                     ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        lib.fmoe_route.argtypes = [ctypes.POINTER(FmoeProblem), ctypes.c_void_p, ctypes.c_void_p,
                                   ctypes.POINTER(FmoeRouteOut), ctypes.c_void_p, ctypes.c_size_t,
                                   ctypes.c_void_p]
        lib.fmoe_read_device_error.argtypes = [ctypes.POINTER(FmoeProblem), ctypes.c_void_p,
                                               ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32)]
        lib.fmoe_plan_view_get.argtypes = [ctypes.POINTER(FmoeProblem), ctypes.c_void_p,
                                           ctypes.POINTER(FmoePlanView)]
        lib.fmoe_set_stage_events.argtypes = [ctypes.c_void_p]
        lib.fmoe_selftest_wait_timeout.argtypes = [ctypes.c_uint64,
                                                   ctypes.POINTER(ctypes.c_uint64),
                                                   ctypes.c_void_p]
        lib.fmoe_forward_routed.argtypes = [ctypes.POINTER(FmoeProblem), ctypes.c_void_p,
                                            ctypes.c_void_p, ctypes.POINTER(FmoeTensors),
                                            ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        # the prelaid entry points take the same arguments (assigned after their sources)
        lib.fmoe_forward_prelaid.argtypes = lib.fmoe_forward.argtypes
        lib.fmoe_forward_routed_prelaid.argtypes = lib.fmoe_forward_routed.argtypes
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        lib.fmoe_ep_plan.argtypes = [vp, i64, i32, i32, i32, vp, vp, vp, vp]
        lib.fmoe_ep_plan_placed.argtypes = [vp, i64, i32, i32, i32, vp, i32, vp, vp, vp, vp]
        lib.fmoe_ep_pack.argtypes = [vp, vp, vp, vp, vp, i64, i32, i32, i32, vp, vp]
        lib.fmoe_ep_unpack.argtypes = [vp, i64, i32, i32, vp, vp, vp, vp, vp]
        lib.fmoe_ep_unpack_count.argtypes = [vp, i64, vp, i32, i32, vp, vp, vp, vp, vp]
        lib.fmoe_ep_offsets.argtypes = [vp, i32, i32, vp, vp, vp]
        lib.fmoe_forward_routed_count.argtypes = [ctypes.POINTER(FmoeProblem), vp, vp, vp,
                                                  ctypes.POINTER(FmoeTensors), vp,
                                                  ctypes.c_size_t, vp]
        lib.fmoe_forward_routed_count_p2p.argtypes = [
            ctypes.POINTER(FmoeProblem), vp, vp, vp, ctypes.POINTER(FmoeTensors), vp,
            ctypes.c_size_t, vp, vp, vp, i32, i64, vp, vp]
        lib.fmoe_ep_combine.argtypes = [vp, vp, i64, i32, i32, vp, vp]
        lib.fmoe_ep_ipc_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(vp), vp]
        lib.fmoe_ep_ipc_open.argtypes = [vp, ctypes.POINTER(vp)]
        lib.fmoe_ep_ipc_close.argtypes = [vp]
        lib.fmoe_ep_ipc_free.argtypes = [vp]
        lib.fmoe_ep_pack_p2p.argtypes = [vp, vp, vp, vp, vp, i64, i32, i32, i32, vp, vp, i64, vp,
                                         vp]
        lib.fmoe_ep_return_p2p.argtypes = [vp, i64, i32, i32, vp, vp, vp, i64, vp, vp]
        lib.fmoe_poll_device_error.argtypes = [ctypes.POINTER(ctypes.c_int32)]
        lib.fmoe_selftest_inject_device_error.argtypes = [ctypes.c_int32]
        lib.fmoe_probe_fp8_mma_rate.argtypes = [i64, ctypes.POINTER(ctypes.c_double),
                                                ctypes.POINTER(ctypes.c_double), vp]
        for name in EXPORTED_SYMBOLS:
            if not hasattr(lib, name):
                raise RuntimeError(f"{p} does not export {name}")
        for name in ("fmoe_forward", "fmoe_forward_routed", "fmoe_forward_prelaid",
                     "fmoe_forward_routed_prelaid"):
            if getattr(lib, name).argtypes is None:
                raise RuntimeError(f"{name}: argument types not set")
        if path is None:
            _lib = lib
        return lib


def _raise(lib, rc: int, where: str):
    msg = lib.fmoe_last_error().decode(errors="replace")
    text = f"{where}: {msg}"
    if rc in (FMOE_ERR_VALUE, FMOE_ERR_WORKSPACE):
        raise ValueError(text)
    if rc == FMOE_ERR_TYPE:
        raise TypeError(text)
    raise RuntimeError(text)


class DeviceError(RuntimeError):
    """A kernel of an earlier (or, with ``check=True``, this) call reported a device error
    word: a bounded wait inside a GEMM ran out, so that call's output is invalid."""


def poll_device_error(device=None) -> int:
    """Error bits reported by calls on ``device`` that finished since the last poll (0 =
    none); does not synchronise (fmoe_poll_device_error)."""
    lib = load_library()
    bits = ctypes.c_int32(0)
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device) \
        if not isinstance(device, torch.device) else device
    with torch.cuda.device(dev):
        rc = lib.fmoe_poll_device_error(ctypes.byref(bits))
    if rc != FMOE_OK:
        _raise(lib, rc, "poll_device_error")
    return int(bits.value)


def _raise_device_error(dev, when: str):
    bits = poll_device_error(dev)
    if bits:
        raise DeviceError(f"{when}: the fused MoE kernels on {dev} reported device error "
                          f"0x{bits:x} (a bounded wait expired); that call's output is invalid")


def inject_device_error(bits: int) -> None:
    """Test hook: the next forward call on this thread reports ``bits`` as its device error
    word (fmoe_selftest_inject_device_error); nothing faults or waits."""
    load_library().fmoe_selftest_inject_device_error(int(bits))


def make_problem(T, E, E_local, H, I, local_expert_offset=0, routed_scaling_factor=2.5,
                 n_group=None, topk_group=None, top_k=None, tile_n=0) -> FmoeProblem:
    if n_group is None or topk_group is None or top_k is None:
        if E not in ROUTING_BY_EXPERTS:
            raise ValueError(f"routing_logits: unsupported number of experts {E}")
        ng, kg, k = ROUTING_BY_EXPERTS[E]
        n_group = ng if n_group is None else n_group
        topk_group = kg if topk_group is None else topk_group
        top_k = k if top_k is None else top_k
    return FmoeProblem(int(T), int(E), int(E_local), int(H), int(I), int(top_k), int(n_group),
                       int(topk_group), int(local_expert_offset), float(routed_scaling_factor),
                       int(tile_n))


def tile_n(prob: FmoeProblem) -> int:
    """Token tile a call with this problem uses (fmoe_tile_n)."""
    lib = load_library()
    v = lib.fmoe_tile_n(ctypes.byref(prob))
    if v < 0:
        _raise(lib, -v, "tile_n")
    return v


def workspace_bytes(prob: FmoeProblem) -> int:
    lib = load_library()
    n = ctypes.c_size_t(0)
    rc = lib.fmoe_workspace_size(ctypes.byref(prob), ctypes.byref(n))
    if rc != FMOE_OK:
        _raise(lib, rc, "workspace_size")
    return int(n.value)


class Workspace:
    """Grow-only device scratch buffer, one per device (the reference keeps thread-local
    grow-only caches for the same purpose, kernel.cu:234-270)."""

    _per_device: dict = {}
    _lock = threading.Lock()

    @classmethod
    def get(cls, device: torch.device, nbytes: int) -> torch.Tensor:
        key = (device.type, device.index)
        with cls._lock:
            buf = cls._per_device.get(key)
            if buf is None or buf.numel() < nbytes:
                buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
                cls._per_device[key] = buf
            return buf


_F32, _BF16, _F8 = torch.float32, torch.bfloat16, torch.float8_e4m3fn


def _check_tensor(t, name, shape, dtype):
    if not isinstance(t, torch.Tensor):
        raise ValueError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if t.dim() != len(shape):
        raise ValueError(f"{name} must be {len(shape)}D, got {t.dim()}")
    for i, (got, exp) in enumerate(zip(t.shape, shape)):
        if got != exp:
            raise ValueError(f"{name} shape mismatch at dim {i}: expected {exp}, got {got}")
    if t.dtype != dtype:
        raise TypeError(f"{name} dtype mismatch: expected {dtype}, got {t.dtype}")


def _validate(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
              gemm1_weights_scale, gemm2_weights, gemm2_weights_scale):
    """Tensor contract of kernel.cu:1746-1769 with geometry derived from the shapes."""
    if not isinstance(routing_logits, torch.Tensor) or routing_logits.dim() != 2:
        raise ValueError("routing_logits must be 2D")
    if not isinstance(gemm1_weights, torch.Tensor) or gemm1_weights.dim() != 3:
        raise ValueError("gemm1_weights must be 3D")
    T, E = routing_logits.shape
    EL, two_i, H = gemm1_weights.shape
    I = two_i // 2
    if H % 128 or I % 128 or H == 0 or I == 0:
        raise ValueError("gemm1_weights: hidden and intermediate sizes must be multiples of 128")
    _check_tensor(routing_logits, "routing_logits", (T, E), _F32)
    _check_tensor(routing_bias, "routing_bias", (E,), _BF16)
    _check_tensor(hidden_states, "hidden_states", (T, H), _F8)
    _check_tensor(hidden_states_scale, "hidden_states_scale", (H // 128, T), _F32)
    _check_tensor(gemm1_weights, "gemm1_weights", (EL, 2 * I, H), _F8)
    _check_tensor(gemm1_weights_scale, "gemm1_weights_scale", (EL, 2 * I // 128, H // 128), _F32)
    _check_tensor(gemm2_weights, "gemm2_weights", (EL, H, I), _F8)
    _check_tensor(gemm2_weights_scale, "gemm2_weights_scale", (EL, H // 128, I // 128), _F32)
    dev = routing_logits.device
    for name, t in (("routing_bias", routing_bias), ("hidden_states", hidden_states),
                    ("hidden_states_scale", hidden_states_scale), ("gemm1_weights", gemm1_weights),
                    ("gemm1_weights_scale", gemm1_weights_scale), ("gemm2_weights", gemm2_weights),
                    ("gemm2_weights_scale", gemm2_weights_scale)):
        if t.device != dev:
            raise ValueError(f"routing_logits and {name} must be on the same device")
    return T, E, EL, H, I


def kernel(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
           gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset: int,
           routed_scaling_factor: float, *, out: torch.Tensor | None = None, tile_n: int = 0,
           workspace: torch.Tensor | None = None, routing: tuple | None = None,
           check: bool = False, prelaid: bool = False) -> torch.Tensor:
    """Fused FP8 block-scaled DeepSeek-V3 MoE layer; returns bf16 [T, H].

    Same positional signature as the reference ``kernel`` (kernel.cu:1727-1734). Extra
    keyword-only arguments: ``out`` (destination), ``tile_n`` (override the autotune
    table), ``workspace`` (caller scratch), ``routing`` ((n_group, topk_group, top_k)
    override), ``check`` (synchronise the stream and raise ``DeviceError`` if this call's
    kernels reported a device error, as the reference's final synchronisation would,
    kernel.cu:1834), ``prelaid`` (the weight tensors are ``prelayout_weights`` outputs).
    Work is enqueued on the current torch stream; without ``check`` there
    is no host synchronisation, and a device error of an earlier call on the device raises
    ``DeviceError`` (a ``RuntimeError``) at the start of the next call.
    """
    T, E, EL, H, I = _validate(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                               gemm1_weights, gemm1_weights_scale, gemm2_weights,
                               gemm2_weights_scale)
    lib = load_library()
    ng, kg, k = routing if routing is not None else (None, None, None)
    prob = make_problem(T, E, EL, H, I, local_expert_offset, routed_scaling_factor, ng, kg, k,
                        tile_n)
    rc = lib.fmoe_validate(ctypes.byref(prob))
    if rc != FMOE_OK:
        _raise(lib, rc, "kernel")
    dev = routing_logits.device
    _raise_device_error(dev, "an earlier call on this device")
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    else:
        _check_tensor(out, "out", (T, H), _BF16)
    if T == 0:
        return out
    nbytes = workspace_bytes(prob)
    if workspace is None:
        with torch.cuda.device(dev):
            workspace = Workspace.get(dev, nbytes)
    tens = FmoeTensors(routing_logits.data_ptr(), routing_bias.data_ptr(),
                       hidden_states.data_ptr(), hidden_states_scale.data_ptr(),
                       gemm1_weights.data_ptr(), gemm1_weights_scale.data_ptr(),
                       gemm2_weights.data_ptr(), gemm2_weights_scale.data_ptr(), out.data_ptr())
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        fwd = lib.fmoe_forward_prelaid if prelaid else lib.fmoe_forward
        rc = fwd(ctypes.byref(prob), ctypes.byref(tens), workspace.data_ptr(), workspace.numel(),
                 stream)
    if rc != FMOE_OK:
        _raise(lib, rc, "kernel")
    if check:
        torch.cuda.current_stream(dev).synchronize()
        _raise_device_error(dev, "this call")
    return out


def forward_routed(topk_idx, topk_w, hidden_states, hidden_states_scale, gemm1_weights,
                   gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                   local_expert_offset: int, num_experts: int = 256, *, out=None,
                   tile_n: int = 0, n_group=None, topk_group=None,
                   check: bool = False, prelaid: bool = False,
                   num_tokens_dev: torch.Tensor | None = None, return_to=None) -> torch.Tensor:
    """The operator on precomputed routing (``topk_idx`` int32 / ``topk_w`` fp32 [T, K]).

    Returns per-token sums over the local experts [offset, offset + E_local) in bf16.
    With ``num_tokens_dev`` (int32 [1] on the device) T is a capacity and only the first
    ``num_tokens_dev[0]`` tokens are processed (fmoe_forward_routed_count); the output rows
    past them are left as they were. ``return_to=(peers, src_start, row_shift, capacity_rows,
    err)`` (with ``num_tokens_dev``) writes each output row straight into its source rank's
    return buffer instead of ``out`` (fmoe_forward_routed_count_p2p).
    """
    T, K = topk_idx.shape
    EL, two_i, H = gemm1_weights.shape
    I = two_i // 2
    _check_tensor(topk_idx, "topk_idx", (T, K), torch.int32)
    _check_tensor(topk_w, "topk_w", (T, K), _F32)
    _check_tensor(hidden_states, "hidden_states", (T, H), _F8)
    _check_tensor(hidden_states_scale, "hidden_states_scale", (H // 128, T), _F32)
    _check_tensor(gemm1_weights, "gemm1_weights", (EL, 2 * I, H), _F8)
    _check_tensor(gemm1_weights_scale, "gemm1_weights_scale", (EL, 2 * I // 128, H // 128), _F32)
    _check_tensor(gemm2_weights, "gemm2_weights", (EL, H, I), _F8)
    _check_tensor(gemm2_weights_scale, "gemm2_weights_scale", (EL, H // 128, I // 128), _F32)
    lib = load_library()
    ng, kg, _ = ROUTING_BY_EXPERTS.get(num_experts, (n_group, topk_group, K))
    prob = make_problem(T, num_experts, EL, H, I, local_expert_offset, 1.0,
                        n_group or ng, topk_group or kg, K, tile_n)
    dev = hidden_states.device
    _raise_device_error(dev, "an earlier call on this device")
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    if T == 0:
        return out
    nbytes = workspace_bytes(prob)
    ws = Workspace.get(dev, nbytes)
    tens = FmoeTensors(0, 0, hidden_states.data_ptr(), hidden_states_scale.data_ptr(),
                       gemm1_weights.data_ptr(), gemm1_weights_scale.data_ptr(),
                       gemm2_weights.data_ptr(), gemm2_weights_scale.data_ptr(), out.data_ptr())
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        if num_tokens_dev is not None:
            if prelaid:
                raise ValueError("forward_routed: num_tokens_dev with prelaid weights is not "
                                 "supported")
            _check_tensor(num_tokens_dev, "num_tokens_dev", (1,), torch.int32)
            if return_to is not None:
                peers, src_start, row_shift, cap_rows, err = return_to
                rc = lib.fmoe_forward_routed_count_p2p(
                    ctypes.byref(prob), topk_idx.data_ptr(), topk_w.data_ptr(),
                    num_tokens_dev.data_ptr(), ctypes.byref(tens), ws.data_ptr(), ws.numel(),
                    peers.back_ptrs.data_ptr(), src_start.data_ptr(), row_shift.data_ptr(),
                    row_shift.shape[0], cap_rows, err.data_ptr(), stream)
            else:
                rc = lib.fmoe_forward_routed_count(ctypes.byref(prob), topk_idx.data_ptr(),
                                                   topk_w.data_ptr(), num_tokens_dev.data_ptr(),
                                                   ctypes.byref(tens), ws.data_ptr(),
                                                   ws.numel(), stream)
        else:
            fwd = lib.fmoe_forward_routed_prelaid if prelaid else lib.fmoe_forward_routed
            rc = fwd(ctypes.byref(prob), topk_idx.data_ptr(), topk_w.data_ptr(),
                     ctypes.byref(tens), ws.data_ptr(), ws.numel(), stream)
    if rc != FMOE_OK:
        _raise(lib, rc, "forward_routed")
    if check:
        torch.cuda.current_stream(dev).synchronize()
        _raise_device_error(dev, "this call")
    return out


def prelayout_weights(gemm1_weights: torch.Tensor, gemm2_weights: torch.Tensor):
    """The weights as the GEMMs load them (fmoe_prelayout_weights): new tensors of the same
    shapes and dtype holding every 128-K weight tile as its swizzled shared-memory image,
    for ``kernel(..., prelaid=True)`` / ``forward_routed(..., prelaid=True)``. The FP8 values
    and the scale tensors are unchanged; done once per set of weights, not per call."""
    EL, two_i, H = gemm1_weights.shape
    I = two_i // 2
    _check_tensor(gemm1_weights, "gemm1_weights", (EL, 2 * I, H), _F8)
    _check_tensor(gemm2_weights, "gemm2_weights", (EL, H, I), _F8)
    lib = load_library()
    prob = make_problem(1, 256, EL, H, I)
    out1 = torch.empty_like(gemm1_weights)
    out2 = torch.empty_like(gemm2_weights)
    dev = gemm1_weights.device
    with torch.cuda.device(dev):
        rc = lib.fmoe_prelayout_weights(ctypes.byref(prob), gemm1_weights.data_ptr(),
                                        gemm2_weights.data_ptr(), out1.data_ptr(),
                                        out2.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    if rc != FMOE_OK:
        _raise(lib, rc, "prelayout_weights")
    return out1, out2


def route(routing_logits: torch.Tensor, routing_bias: torch.Tensor, n_group: int,
          topk_group: int, top_k: int, routed_scaling_factor: float, num_local_experts: int = 1,
          local_expert_offset: int = 0):
    """Routing kernel only: returns (topk_idx int32 [T, K], topk_w fp32 [T, K]) on device."""
    T, E = routing_logits.shape
    _check_tensor(routing_logits, "routing_logits", (T, E), _F32)
    _check_tensor(routing_bias, "routing_bias", (E,), _BF16)
    lib = load_library()
    prob = make_problem(T, E, num_local_experts, 128, 128, local_expert_offset,
                        routed_scaling_factor, n_group, topk_group, top_k)
    dev = routing_logits.device
    idx = torch.empty(T, top_k, dtype=torch.int32, device=dev)
    w = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    if T == 0:
        return idx, w
    nbytes = workspace_bytes(prob)
    ws = Workspace.get(dev, nbytes)
    ro = FmoeRouteOut(idx.data_ptr(), w.data_ptr())
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.fmoe_route(ctypes.byref(prob), routing_logits.data_ptr(), routing_bias.data_ptr(),
                            ctypes.byref(ro), ws.data_ptr(), ws.numel(), stream)
    if rc != FMOE_OK:
        _raise(lib, rc, "route")
    return idx, w


# ---- expert-parallel exchange, device side (include/fmoe.h fmoe_ep_*) ----------------------
def ep_payload_bytes(H: int, K: int) -> int:
    """Bytes of one exchange row: FP8 row | block scales | expert ids | weights."""
    return H + 4 * (H // 128) + 8 * K


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def ep_plan(topk_idx: torch.Tensor, world: int, experts_per_rank: int,
            expert_pos: torch.Tensor | None = None):
    """Send plan: (pos int32 [world, T], tokens int32 [sum], counts int32 [world]).

    With ``expert_pos`` (int32 [world * experts_per_rank] on the device: each expert's
    position in an expert placement) the ids in ``topk_idx`` are first replaced in place by
    their positions (fmoe_ep_plan_placed)."""
    T, K = topk_idx.shape
    dev = topk_idx.device
    lib = load_library()
    pos = torch.empty(world, T, dtype=torch.int32, device=dev)
    tokens = torch.empty(max(T * world, 1), dtype=torch.int32, device=dev)
    counts = torch.empty(world, dtype=torch.int32, device=dev)
    if expert_pos is not None:
        _check_tensor(expert_pos, "expert_pos", (world * experts_per_rank,), torch.int32)
        if not topk_idx.is_contiguous():
            raise ValueError("ep_plan: topk_idx must be contiguous (it is remapped in place)")
        rc = lib.fmoe_ep_plan_placed(topk_idx.data_ptr(), T, K, world, experts_per_rank,
                                     expert_pos.data_ptr(), expert_pos.numel(), pos.data_ptr(),
                                     tokens.data_ptr(), counts.data_ptr(), _stream(dev))
    else:
        rc = lib.fmoe_ep_plan(topk_idx.data_ptr(), T, K, world, experts_per_rank,
                              pos.data_ptr(), tokens.data_ptr(), counts.data_ptr(), _stream(dev))
    if rc != FMOE_OK:
        _raise(lib, rc, "ep_plan")
    return pos, tokens, counts


def ep_pack(hidden_states, hidden_states_scale, topk_idx, topk_w, pos, rows: int):
    """Exchange rows for every (token, rank) of the plan, [rows, payload] uint8."""
    T, H = hidden_states.shape
    K = topk_idx.shape[1]
    dev = hidden_states.device
    lib = load_library()
    send = torch.empty(rows, ep_payload_bytes(H, K), dtype=torch.uint8, device=dev)
    rc = lib.fmoe_ep_pack(hidden_states.data_ptr(), hidden_states_scale.data_ptr(),
                          topk_idx.data_ptr(), topk_w.data_ptr(), pos.data_ptr(), T, H, K,
                          pos.shape[0], send.data_ptr(), _stream(dev))
    if rc != FMOE_OK:
        _raise(lib, rc, "ep_pack")
    return send


def ep_unpack(recv, H: int, K: int, rows: int = None, device=None):
    """Received rows -> (hidden fp8 [R, H], scale fp32 [H/128, R], idx int32, w fp32).
    `recv` is a uint8 tensor of payload rows, or a raw device pointer (int) with `rows` and
    `device` given."""
    if isinstance(recv, int):
        R, dev, ptr = rows, device, recv
    else:
        R, dev, ptr = recv.shape[0], recv.device, recv.data_ptr()
    lib = load_library()
    hs = torch.empty(R, H, dtype=torch.float8_e4m3fn, device=dev)
    sc = torch.empty(H // 128, R, dtype=torch.float32, device=dev)
    idx = torch.empty(R, K, dtype=torch.int32, device=dev)
    w = torch.empty(R, K, dtype=torch.float32, device=dev)
    rc = lib.fmoe_ep_unpack(ptr, R, H, K, hs.data_ptr(), sc.data_ptr(),
                            idx.data_ptr(), w.data_ptr(), _stream(dev))
    if rc != FMOE_OK:
        _raise(lib, rc, "ep_unpack")
    return hs, sc, idx, w


def ep_unpack_count(recv, capacity_rows: int, rows_dev: torch.Tensor, H: int, K: int,
                    out=None, device=None):
    """fmoe_ep_unpack_count: the first rows_dev[0] received rows into arrays sized for
    `capacity_rows` rows -- (hidden fp8 [cap, H], scale fp32 [H/128, cap], idx, w), or into
    `out` (the same four tensors, reused across calls). `recv`: tensor or raw pointer."""
    if isinstance(recv, int):
        dev, ptr = device, recv
    else:
        dev, ptr = recv.device, recv.data_ptr()
    lib = load_library()
    if out is None:
        out = (torch.empty(capacity_rows, H, dtype=torch.float8_e4m3fn, device=dev),
               torch.empty(H // 128, capacity_rows, dtype=torch.float32, device=dev),
               torch.empty(capacity_rows, K, dtype=torch.int32, device=dev),
               torch.empty(capacity_rows, K, dtype=torch.float32, device=dev))
    hs, sc, idx, w = out
    _check_tensor(rows_dev, "rows_dev", (1,), torch.int32)
    rc = lib.fmoe_ep_unpack_count(ptr, capacity_rows, rows_dev.data_ptr(), H, K, hs.data_ptr(),
                                  sc.data_ptr(), idx.data_ptr(), w.data_ptr(), _stream(dev))
    if rc != FMOE_OK:
        _raise(lib, rc, "ep_unpack_count")
    return out


def ep_offsets(counts_all: torch.Tensor, rank: int, tables=None, rows=None):
    """fmoe_ep_offsets: (tables int64 [3 world + 1], rows int32 [1]) on the device from the
    int64 [world, world + 1] all-gather of the ranks' per-destination counts."""
    world = counts_all.shape[0]
    dev = counts_all.device
    _check_tensor(counts_all, "counts_all", (world, world + 1), torch.int64)
    if tables is None:
        tables = torch.empty(3 * world + 1, dtype=torch.int64, device=dev)
    if rows is None:
        rows = torch.empty(1, dtype=torch.int32, device=dev)
    lib = load_library()
    rc = lib.fmoe_ep_offsets(counts_all.data_ptr(), world, rank, tables.data_ptr(),
                             rows.data_ptr(), _stream(dev))
    if rc != FMOE_OK:
        _raise(lib, rc, "ep_offsets")
    return tables, rows


def ep_combine(back, pos: torch.Tensor, T: int, H: int = None):
    """Per token, its returned partial rows summed in fp32 in rank order -> bf16 [T, H].
    `back` is a bf16 tensor [rows, H] or a raw device pointer (int) with `H` given."""
    if isinstance(back, int):
        ptr = back
    else:
        H, ptr = back.shape[1], back.data_ptr()
    dev = pos.device
    lib = load_library()
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    rc = lib.fmoe_ep_combine(ptr, pos.data_ptr(), T, H, pos.shape[0],
                             out.data_ptr(), _stream(dev))
    if rc != FMOE_OK:
        _raise(lib, rc, "ep_combine")
    return out


class PeerBuffers:
    """This rank's receive and return buffers and every peer's, mapped by CUDA IPC.

    Collective: every rank of `group` constructs it with the same sizes (the handles are
    exchanged with all_gather_object). `recv[r]` / `back[r]` hold rank r's buffers as device
    addresses in this process; `recv_ptrs` / `back_ptrs` are the same as device int64 arrays
    for the P2P kernels."""

    def __init__(self, recv_bytes: int, back_bytes: int, group, device):
        import torch.distributed as dist

        lib = load_library()
        self._lib = lib
        self.recv_bytes, self.back_bytes = recv_bytes, back_bytes
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        own = []
        handles = []
        with torch.cuda.device(device):
            for nbytes in (recv_bytes, back_bytes):
                ptr = ctypes.c_void_p()
                h = ctypes.create_string_buffer(64)
                rc = lib.fmoe_ep_ipc_alloc(nbytes, ctypes.byref(ptr), h)
                if rc != FMOE_OK:
                    _raise(lib, rc, "ep_ipc_alloc")
                own.append(ptr.value)
                handles.append(h.raw)
            gathered = [None] * world
            dist.all_gather_object(gathered, handles, group=group)
            self._opened = []
            maps = [[0] * world, [0] * world]
            for r in range(world):
                for which in range(2):
                    if r == rank:
                        maps[which][r] = own[which]
                        continue
                    ptr = ctypes.c_void_p()
                    rc = lib.fmoe_ep_ipc_open(gathered[r][which], ctypes.byref(ptr))
                    if rc != FMOE_OK:
                        _raise(lib, rc, "ep_ipc_open")
                    maps[which][r] = ptr.value
                    self._opened.append(ptr.value)
        self._own = own
        self.recv, self.back = maps
        self.recv_ptrs = torch.tensor(self.recv, dtype=torch.int64, device=device)
        self.back_ptrs = torch.tensor(self.back, dtype=torch.int64, device=device)

    def close(self):
        """Unmap the peers' buffers and free this rank's (after a barrier: no peer may still
        write into them)."""
        for ptr in self._opened:
            self._lib.fmoe_ep_ipc_close(ptr)
        for ptr in self._own:
            self._lib.fmoe_ep_ipc_free(ptr)
        self._opened, self._own = [], []


def ep_pack_p2p(hidden_states, hidden_states_scale, topk_idx, topk_w, pos, peers: PeerBuffers,
                row_shift: torch.Tensor, capacity_rows: int, err: torch.Tensor):
    T, H = hidden_states.shape
    K = topk_idx.shape[1]
    dev = hidden_states.device
    lib = load_library()
    rc = lib.fmoe_ep_pack_p2p(hidden_states.data_ptr(), hidden_states_scale.data_ptr(),
                              topk_idx.data_ptr(), topk_w.data_ptr(), pos.data_ptr(), T, H, K,
                              pos.shape[0], peers.recv_ptrs.data_ptr(), row_shift.data_ptr(),
                              capacity_rows, err.data_ptr(), _stream(dev))
    if rc != FMOE_OK:
        _raise(lib, rc, "ep_pack_p2p")


def ep_return_p2p(partial: torch.Tensor, src_start: torch.Tensor, peers: PeerBuffers,
                  row_shift: torch.Tensor, capacity_rows: int, err: torch.Tensor):
    R, H = partial.shape
    dev = partial.device
    lib = load_library()
    rc = lib.fmoe_ep_return_p2p(partial.data_ptr(), R, H, row_shift.shape[0],
                                src_start.data_ptr(), peers.back_ptrs.data_ptr(),
                                row_shift.data_ptr(), capacity_rows, err.data_ptr(), _stream(dev))
    if rc != FMOE_OK:
        _raise(lib, rc, "ep_return_p2p")


def read_device_error(prob: FmoeProblem, workspace: torch.Tensor) -> int:
    """Synchronise and return (and clear) the device error word of the last call."""
    lib = load_library()
    val = ctypes.c_int32(0)
    stream = torch.cuda.current_stream(workspace.device).cuda_stream
    rc = lib.fmoe_read_device_error(ctypes.byref(prob), workspace.data_ptr(), stream,
                                    ctypes.byref(val))
    if rc != FMOE_OK:
        _raise(lib, rc, "read_device_error")
    return int(val.value)


def selftest_wait_timeout(timeout_ns: int = 2_000_000, device=None) -> dict:
    """Run the bounded-wait self-test kernel on the current stream: both of its waits can
    never complete and must expire after ``timeout_ns``. Returns which expired and how
    long each waited (ns); raises if the kernel itself failed."""
    lib = load_library()
    res = (ctypes.c_uint64 * 3)()
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.fmoe_selftest_wait_timeout(int(timeout_ns), res, stream)
    if rc != FMOE_OK:
        _raise(lib, rc, "selftest_wait_timeout")
    return {"expired_mask": int(res[0]), "mbarrier_wait_ns": int(res[1]),
            "flag_wait_ns": int(res[2])}


def probe_fp8_mma_rate(mmas_per_cta: int = 16384, device=None) -> dict:
    """Measured dense FP8 tensor-core rate of the current GPU (fmoe_probe_fp8_mma_rate):
    {"tflops": dense TFLOP/s, "ms": time of the timed launch}."""
    lib = load_library()
    tf, ms = ctypes.c_double(0.0), ctypes.c_double(0.0)
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    with torch.cuda.device(dev):
        rc = lib.fmoe_probe_fp8_mma_rate(int(mmas_per_cta), ctypes.byref(tf), ctypes.byref(ms),
                                         torch.cuda.current_stream(dev).cuda_stream)
    if rc != FMOE_OK:
        _raise(lib, rc, "probe_fp8_mma_rate")
    return {"tflops": tf.value, "ms": ms.value}


def plan_view(prob: FmoeProblem, workspace: torch.Tensor) -> dict:
    """Copies of the permutation the last call built (expert counts/offsets, row maps)."""
    lib = load_library()
    v = FmoePlanView()
    rc = lib.fmoe_plan_view_get(ctypes.byref(prob), workspace.data_ptr(), ctypes.byref(v))
    if rc != FMOE_OK:
        _raise(lib, rc, "plan_view")
    base = workspace.data_ptr()
    w32 = workspace.view(torch.int32) if workspace.numel() % 4 == 0 else None

    def grab(ptr, n):
        off = (ptr - base) // 4
        return w32[off:off + n].clone()

    T, K, EL = prob.num_tokens, prob.top_k, prob.num_local_experts
    return dict(expert_cnt=grab(v.expert_cnt, EL), expert_off=grab(v.expert_off, EL + 1),
                row_token=grab(v.row_token, v.row_cap), token_row=grab(v.token_row, T * K),
                meta=grab(v.meta, 16), row_cap=int(v.row_cap))


class StageTimer:
    """Records CUDA events at the six stage boundaries of every fmoe_forward() on this
    thread (see fmoe_set_stage_events in include/fmoe.h); ``times_ms()`` returns the five
    stage durations of the most recent call: route, permute, gemm1, gemm2, combine."""

    STAGES = ("route", "permute", "gemm1", "gemm2", "combine")

    def __init__(self):
        self.events = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
        for e in self.events:  # torch creates the CUDA event lazily, on first record
            e.record()
        self._arr = (ctypes.c_void_p * 6)(*[e.cuda_event for e in self.events])

    def __enter__(self):
        lib = load_library()
        rc = lib.fmoe_set_stage_events(ctypes.cast(self._arr, ctypes.c_void_p))
        if rc != FMOE_OK:
            _raise(lib, rc, "set_stage_events")
        return self

    def __exit__(self, *exc):
        load_library().fmoe_set_stage_events(None)
        return False

    def times_ms(self):
        return [self.events[i].elapsed_time(self.events[i + 1]) for i in range(5)]


def load_tvm_ffi_kernel():
    """The TVM-FFI `kernel` export (reference binding "tvm-ffi", kernel.cu:1839)."""
    import tvm_ffi

    load_library()
    if not TVM_FFI_LIB_PATH.exists():
        raise RuntimeError(f"TVM-FFI binding not built: {TVM_FFI_LIB_PATH}")
    mod = tvm_ffi.load_module(str(TVM_FFI_LIB_PATH))
    return mod["kernel"]
