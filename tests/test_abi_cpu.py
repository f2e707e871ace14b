"""CPU checks of the C ABI: the library loads, exports every function include/fmoe.h
declares, and rejects bad arguments with the reference's error classes -- all without
a GPU (no compute call is made)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent


def header_functions():
    text = (ROOT / "include" / "fmoe.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(fmoe_\w+)\s*\(", text, re.M)))


def test_library_exports_header(fmoe):
    lib = fmoe.load_library()
    names = header_functions()
    assert len(names) >= 9
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(fmoe.EXPORTED_SYMBOLS)
    assert lib.fmoe_abi_version() == 1


def test_tvm_ffi_binding_exports_kernel(fmoe):
    lib = ctypes.CDLL(str(fmoe.TVM_FFI_LIB_PATH))
    assert hasattr(lib, "__tvm_ffi_kernel")


def _prob(fmoe, **kw):
    base = dict(T=16, E=256, E_local=32, H=7168, I=2048)
    base.update(kw)
    return fmoe.make_problem(base["T"], base["E"], base["E_local"], base["H"], base["I"])


@pytest.mark.parametrize("field,value", [
    ("num_tokens", -1), ("num_experts", 0), ("num_experts", 512), ("n_group", 7),
    ("topk_group", 9), ("top_k", 0), ("top_k", 33), ("num_local_experts", 257),
    ("hidden_size", 100), ("intermediate_size", 64), ("tile_n", 48)])
def test_validate_rejects(fmoe, field, value):
    lib = fmoe.load_library()
    p = _prob(fmoe)
    setattr(p, field, value)
    assert lib.fmoe_validate(ctypes.byref(p)) == fmoe.FMOE_ERR_VALUE
    assert len(lib.fmoe_last_error()) > 0


def test_validate_accepts_both_geometries(fmoe):
    lib = fmoe.load_library()
    assert lib.fmoe_validate(ctypes.byref(_prob(fmoe))) == fmoe.FMOE_OK
    tiny = fmoe.make_problem(16, 16, 16, 256, 128)
    assert (tiny.n_group, tiny.topk_group, tiny.top_k) == (4, 2, 4)
    assert lib.fmoe_validate(ctypes.byref(tiny)) == fmoe.FMOE_OK


def test_validate_throughput_tile_needs_hidden_multiple_of_256(fmoe):
    lib = fmoe.load_library()
    p = _prob(fmoe, T=4096)
    p.tile_n = 128
    assert lib.fmoe_validate(ctypes.byref(p)) == fmoe.FMOE_OK
    odd = fmoe.make_problem(64, 16, 16, 384, 128)
    odd.tile_n = 128
    assert lib.fmoe_validate(ctypes.byref(odd)) == fmoe.FMOE_ERR_VALUE
    assert b"multiple of 256" in lib.fmoe_last_error()
    odd.tile_n = 0  # the table's 128 falls back to the decode family instead
    assert lib.fmoe_validate(ctypes.byref(odd)) == fmoe.FMOE_OK


def test_workspace_size_grows_with_tokens(fmoe):
    sizes = [fmoe.workspace_bytes(_prob(fmoe, T=t)) for t in (1, 64, 4096)]
    assert sizes[0] < sizes[1] < sizes[2]
    assert sizes[2] > 4096 * 7168  # holds at least the permuted FP8 rows


def test_autotune_table(fmoe):
    lib = fmoe.load_library()
    tiles = [lib.fmoe_autotune_tile_n(t) for t in (1, 64, 256, 512, 2048, 4096, 8192)]
    assert all(t in (16, 32, 64, 128, 256) for t in tiles)
    assert tiles == sorted(tiles)
    # DeepSeek-V3 routing: the bounds of 8 and 24 expected rows per local expert
    assert [lib.fmoe_autotune_tile_n(t) for t in (256, 257, 768, 769)] == [16, 64, 64, 128]


def test_tile_follows_rows_per_expert(fmoe):
    """The table is keyed by T * top_k / E_global: the DS-V3 slice, the whole 256-expert
    layer and the 16-expert geometry reach the same tile at the same rows per expert."""
    dsv3 = [fmoe.tile_n(fmoe.make_problem(t, 256, e, 7168, 2048)) for t in (256, 257, 769)
            for e in (32, 256)]
    assert dsv3 == [16, 16, 64, 64, 128, 128]
    # 16 experts, top_k 4: 8 rows per expert at 32 tokens, 24 at 96
    tiny = [fmoe.tile_n(fmoe.make_problem(t, 16, 16, 256, 128)) for t in (32, 33, 96, 97)]
    assert tiny == [16, 64, 64, 128]
    # the throughput family needs hidden_size % 256 == 0; otherwise 64
    assert fmoe.tile_n(fmoe.make_problem(97, 16, 16, 384, 128)) == 64
    assert fmoe.tile_n(fmoe.make_problem(1, 256, 32, 7168, 2048, tile_n=32)) == 32
    with pytest.raises(ValueError):
        fmoe.tile_n(fmoe.make_problem(1, 256, 32, 100, 2048))


def test_forward_rejects_null_and_empty_without_gpu(fmoe):
    lib = fmoe.load_library()
    p = _prob(fmoe)
    t = fmoe.FmoeTensors()
    rc = lib.fmoe_forward(ctypes.byref(p), ctypes.byref(t), None, 0, None)
    assert rc == fmoe.FMOE_ERR_VALUE
    assert b"must not be NULL" in lib.fmoe_last_error()
    p0 = _prob(fmoe, T=0)
    assert lib.fmoe_forward(ctypes.byref(p0), ctypes.byref(t), None, 0, None) == fmoe.FMOE_OK


def test_python_kernel_rejects_cpu_tensors(fmoe):
    from fmoe_b200 import workloads as W

    inp = W.make_inputs(W.TINY, 4, seed=0)
    with pytest.raises(ValueError, match="must be a CUDA tensor"):
        fmoe.kernel(*W.operator_args(inp), 0, 2.5)
    args = W.operator_args(inp)
    args[0] = args[0][:, :8]
    with pytest.raises(ValueError):
        fmoe.kernel(*args, 0, 2.5)


def test_python_kernel_rejects_unknown_expert_count(fmoe):
    with pytest.raises(ValueError, match="unsupported number of experts"):
        fmoe.make_problem(4, 24, 8, 256, 128)
