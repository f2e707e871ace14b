"""flashinfer-bench packaging (fused-moe-yws_b200/pack_solution.py): the solution.json
follows the reference packer's schema, carries every library source verbatim, and its
entry point names a file that exports the TVM-FFI function."""
import json
import re
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "fused-moe-yws_b200"


def test_pack_solution_schema_and_sources(tmp_path):
    out = tmp_path / "solution.json"
    subprocess.check_call([sys.executable, str(PKG / "pack_solution.py"), "-o", str(out)])
    sol = json.loads(out.read_text())
    assert set(sol) == {"name", "definition", "author", "spec", "sources", "description"}
    assert sol["definition"] == "moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048"
    spec = sol["spec"]
    assert spec["language"] == "cuda" and spec["binding"] == "tvm-ffi"
    assert spec["destination_passing_style"] is False
    paths = {s["path"]: s["content"] for s in sol["sources"]}
    for f in list((PKG / "csrc").glob("*.cu")) + list((PKG / "csrc").glob("*.cuh")):
        assert paths[f.name] == f.read_text()
    assert paths["fmoe.h"] == (ROOT / "include" / "fmoe.h").read_text()
    entry_file, entry_fn = spec["entry_point"].split("::")
    assert re.search(rf"TVM_FFI_DLL_EXPORT_TYPED_FUNC\(\s*{entry_fn}\s*,", paths[entry_file])
    # every quoted include of a packed source resolves inside the packed tree
    for name, text in paths.items():
        for inc in re.findall(r'#include "([^"]+)"', text):
            assert inc in paths, f"{name} includes {inc}, which is not packed"
