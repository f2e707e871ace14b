"""Pack this library as a flashinfer-bench solution (solution.json).

Same schema as the reference's packer (scripts/pack_solution.py:32-90): name, definition,
author, spec {language, target_hardware, entry_point, destination_passing_style, binding,
dependencies}, sources [{path, content}], description. Metadata comes from
solution.toml beside this file. The sources are every file of csrc/ (kernels, the C ABI,
the TVM-FFI export named by the entry point) plus include/fmoe.h, all at the top level of
the packed tree, so `#include "fmoe.h"` resolves there as it does through `-I include`
in build.py. The kernels use sm_100a instructions (tcgen05, TMA): the consuming harness
must compile with `-gencode arch=compute_100a,code=sm_100a`.

    python fused-moe-yws_b200/pack_solution.py -o solution.json
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

try:
    import tomllib
except ImportError:  # pragma: no cover
    import tomli as tomllib

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
HEADER = PKG.parent / "include" / "fmoe.h"
SOURCE_SUFFIXES = (".cu", ".cuh", ".h", ".cc")


def source_files() -> list[Path]:
    files = sorted(p for p in CSRC.iterdir() if p.is_file() and p.suffix in SOURCE_SUFFIXES)
    return files + [HEADER]


def pack(config_path: Path = PKG / "solution.toml") -> dict:
    cfg = tomllib.loads(config_path.read_text())
    sol, build = cfg["solution"], cfg["build"]
    spec = {
        "language": build["language"],
        "target_hardware": ["cuda"],
        "entry_point": build["entry_point"],
        "destination_passing_style": build.get("destination_passing_style", False),
        "binding": build.get("binding", "tvm-ffi"),
        "dependencies": build.get("dependencies", []),
    }
    sources = [{"path": p.name, "content": p.read_text()} for p in source_files()]
    entry_file = spec["entry_point"].split("::")[0]
    if entry_file not in {s["path"] for s in sources}:
        raise FileNotFoundError(f"entry point file {entry_file} is not among the sources")
    return {"name": sol["name"], "definition": sol["definition"], "author": sol["author"],
            "spec": spec, "sources": sources, "description": sol.get("description", "")}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("-o", "--output", type=Path, default=Path("solution.json"))
    args = ap.parse_args()
    solution = pack()
    args.output.write_text(json.dumps(solution, indent=2))
    print(f"packed {len(solution['sources'])} sources into {args.output} "
          f"(entry point {solution['spec']['entry_point']})")


if __name__ == "__main__":
    main()
