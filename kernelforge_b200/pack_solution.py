"""Pack the CUDA implementation into a flashinfer-bench ``Solution`` JSON.

    python -m kernelforge_b200.pack_solution [-o solution.json] [--name N] [--author A]

The reference's packer (``scripts/pack_solution.py:113-204``, driven by
``config.toml``) writes ``{name, definition, author, spec, sources}`` where
``spec`` carries ``language``, ``target_hardware``, ``entry_point``
(``"<relative file>::<function>"``), ``dependencies``, the optional ``binding``
and ``destination_passing_style``, and ``sources`` is a list of
``{"path", "content"}`` text files.  This packer emits the same layout for the
CUDA build: language ``"cuda"``, binding ``"torch"`` (the reference's
``README.md:404-424`` lists ``"tvm-ffi"`` and ``"torch"`` as CUDA bindings), value-returning style
(``destination_passing_style: false``, as the reference's ``kernel`` returns
its output), and the entry point ``kernelforge_b200/binding.py::kernel`` whose
ten positional parameters are the reference's.

The sources are exactly what the entry point needs: the Python binding and its
build step, the CUDA sources, the PyTorch C++ extension over the C ABI and the
C-ABI header.  On first call the binding compiles ``libkf_moe.so`` for sm_100a
and the extension ``_kf_torch.so`` from them (``build.py``); it has no CPU
fallback.  How the contest harness's own CUDA builder treats these
sources is not known here (the harness is not available), so the JSON is
checked by round-tripping it: unpacked into an empty directory, the sources
build and the entry point imports.
"""
from __future__ import annotations

import argparse
import json
import os
from typing import Dict, List

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)

# The fused_moe track definition the reference targets (its config.toml).
DEFINITION = "moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048"
ENTRY_POINT = "kernelforge_b200/binding.py::kernel"
PY_SOURCES = ["__init__.py", "binding.py", "build.py"]


def source_files() -> List[str]:
    """Repository-relative paths of every file the packed solution carries."""
    from . import build
    files = [os.path.join("kernelforge_b200", f) for f in PY_SOURCES]
    files += [os.path.join("kernelforge_b200", "csrc", f) for f in build.SOURCES + build.HEADERS + [build.EXT_SOURCE]]
    files.append(os.path.join("include", "kf_moe.h"))
    return files


def solution_dict(name: str = "kernelforge-b200", author: str = "kernelforge-b200") -> Dict:
    sources = []
    for rel in source_files():
        with open(os.path.join(ROOT, rel), encoding="utf-8") as f:
            sources.append({"path": rel.replace(os.sep, "/"), "content": f.read()})
    spec = {
        "language": "cuda",
        "target_hardware": ["cuda"],
        "entry_point": ENTRY_POINT,
        "dependencies": [],
        "binding": "torch",
        "destination_passing_style": False,
    }
    return {"name": name, "definition": DEFINITION, "author": author, "spec": spec, "sources": sources}


def unpack(solution: Dict, dest: str) -> None:
    """Write a solution's sources under ``dest`` (used to check a packed file)."""
    for s in solution["sources"]:
        path = os.path.normpath(os.path.join(dest, s["path"]))
        if not path.startswith(os.path.abspath(dest) + os.sep):
            raise ValueError(f"source path escapes the destination: {s['path']}")
        os.makedirs(os.path.dirname(path), exist_ok=True)
        with open(path, "w", encoding="utf-8") as f:
            f.write(s["content"])


def main(argv=None) -> str:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("-o", "--output", default=os.path.join(ROOT, "solution.json"))
    ap.add_argument("--name", default="kernelforge-b200")
    ap.add_argument("--author", default="kernelforge-b200")
    args = ap.parse_args(argv)
    sol = solution_dict(args.name, args.author)
    with open(args.output, "w", encoding="utf-8") as f:
        json.dump(sol, f, indent=2)
    print(f"Solution packed: {args.output} ({len(sol['sources'])} sources, entry {sol['spec']['entry_point']})")
    return args.output


if __name__ == "__main__":
    main()
