"""The packed flashinfer-bench Solution JSON: layout, entry point and a build round trip (CPU only).

Layout follows the reference's packer (``scripts/pack_solution.py:113-204``).
"""
import ast
import json
import os
import shutil
import subprocess
import sys

import pytest

from kernelforge_b200 import pack_solution as P

REF_PARAMS = ["routing_logits", "routing_bias", "hidden_states", "hidden_states_scale", "gemm1_weights",
              "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale", "local_expert_offset",
              "routed_scaling_factor"]


def test_solution_layout(tmp_path):
    out = P.main(["-o", str(tmp_path / "solution.json"), "--name", "t", "--author", "a"])
    sol = json.loads(open(out).read())
    assert set(sol) == {"name", "definition", "author", "spec", "sources"}
    assert sol["definition"] == P.DEFINITION
    spec = sol["spec"]
    assert spec["language"] == "cuda" and spec["binding"] == "torch"
    assert spec["destination_passing_style"] is False and spec["target_hardware"] == ["cuda"]
    paths = {s["path"] for s in sol["sources"]}
    entry_file, fn = spec["entry_point"].split("::")
    assert entry_file in paths and fn == "kernel"
    assert "include/kf_moe.h" in paths
    assert all(s["content"] for s in sol["sources"])


def test_entry_point_signature_matches_reference():
    sol = P.solution_dict()
    entry_file, fn = sol["spec"]["entry_point"].split("::")
    src = next(s["content"] for s in sol["sources"] if s["path"] == entry_file)
    node = next(n for n in ast.parse(src).body if isinstance(n, ast.FunctionDef) and n.name == fn)
    assert [a.arg for a in node.args.args] == REF_PARAMS
    assert node.args.vararg is None and node.args.kwarg is None   # variadic signatures fail the builder check
    assert any(isinstance(n, ast.Return) and n.value is not None for n in ast.walk(node))  # value-returning


def test_unpack_rejects_escaping_paths(tmp_path):
    with pytest.raises(ValueError):
        P.unpack({"sources": [{"path": "../evil.py", "content": "x"}]}, str(tmp_path))


@pytest.mark.skipif(not os.path.exists(os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")), reason="needs nvcc")
def test_unpacked_sources_build_and_import(tmp_path):
    """The sources alone rebuild libkf_moe.so for sm_100a and its torch extension, and the entry point
    imports (no GPU needed)."""
    P.unpack(P.solution_dict(), str(tmp_path))
    code = ("import sys; sys.path.insert(0, '.'); from kernelforge_b200 import build; "
            "build.build(force=True); build.build_ext(force=True); import kernelforge_b200.binding as b; "
            "lib = b.library(); ext = b.extension(); "
            "print(callable(b.kernel) and callable(ext.kernel), lib.kf_moe_launches_per_forward())")
    r = subprocess.run([sys.executable, "-c", code], cwd=tmp_path, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.split()[-2:] == ["True", "7"]
    shutil.rmtree(tmp_path / "kernelforge_b200")
