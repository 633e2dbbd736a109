"""The C-ABI library builds for sm_100a, loads without a GPU, and exports
every entry point include/pse.h declares.  No kernel is launched.  CPU only."""
from __future__ import annotations

import os
import re
import subprocess

import pytest

from conftest import ROOT


def _declared():
    with open(os.path.join(ROOT, "include", "pse.h")) as f:
        text = f.read()
    return sorted(set(re.findall(r"^(?:int|size_t)\s+(pse_\w+)\s*\(", text, flags=re.M)))


def test_library_builds_and_exports_every_declared_symbol():
    from pse import _build, _native
    lib_path = _build.build()
    assert os.path.exists(lib_path)
    lib = _native.load(require_cuda=False)
    declared = _declared()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(lib, name), name
    nm = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT\s+(pse_\w+)", nm))
    assert set(declared) <= exported
    # the ctypes prototype table covers the header exactly
    assert set(_native.exported_symbols()) == set(declared)


def test_ctypes_prototypes_match_the_header():
    """Every prototype in the ctypes table takes as many arguments as the
    header's declaration (a drifted binding would pass misread arguments)."""
    from pse import _native
    with open(os.path.join(ROOT, "include", "pse.h")) as f:
        text = re.sub(r"/\*.*?\*/", "", f.read(), flags=re.S)
    decls = dict(re.findall(r"(?:int|size_t)\s+(pse_\w+)\s*\(([^)]*)\)\s*;", text))
    assert len(decls) == len(_declared())
    checked = 0
    for name, (argtypes, _) in _native._PROTOS.items():
        params = decls[name].strip()
        n = 0 if params in ("", "void") else params.count(",") + 1
        assert len(argtypes) == n, name
        checked += 1
    assert checked >= 20


def test_engine_refuses_to_run_without_cuda():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import pse
    with pytest.raises(RuntimeError):
        pse.PagedKVCache(1, 1, 2, 4, 8)


def test_tensor_map_cache_compares_the_full_descriptor_key(tmp_path):
    """Two pools whose (pointer, sizes) fold onto one 64-bit value still get
    distinct descriptor-cache keys: a hit needs every field equal."""
    cuda_inc = "/usr/local/cuda/include"
    if not os.path.isdir(cuda_inc):
        pytest.skip("CUDA headers not found")
    exe = str(tmp_path / "tmap_key_check")
    src = os.path.join(ROOT, "tests", "native", "tmap_key_check.cpp")
    csrc = os.path.join(ROOT, "paged-speculative-engine_b200", "csrc")
    subprocess.run(["g++", "-std=c++17", "-O1", f"-I{csrc}", f"-I{cuda_inc}", src, "-o", exe], check=True)
    out = subprocess.run([exe], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.strip() == "OK"
