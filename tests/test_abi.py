"""The C-ABI library loads and exports exactly what include/vdx_sampler.h declares.
No compute calls are made here (these run without a GPU)."""
import ctypes as C
import os
import re
import subprocess

import pytest

from vindexllm_b200 import _lib, abi
from vindexllm_b200.build import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "vdx_sampler.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"VDXS_API\s+[\w\s\*]+?\b(vdxs_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.load()


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "vdxs_sample" in syms and "vdxs_sample_sharded" in syms and len(syms) >= 25


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing
    extra = [s for s in exported if s.startswith("vdxs_") and s not in declared_symbols()]
    assert not extra, extra
    assert set(_lib.SIGNATURES) == set(declared_symbols())


def test_exports_are_only_the_abi(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert all(s.startswith("vdxs_") for s in exported), sorted(s for s in exported if not s.startswith("vdxs_"))


def test_config_layout_matches_pascal_record():
    # TVdxSamplerConfig under {$A8}: offsets 0,4,8,12,16,20,24; size 32.
    assert C.sizeof(abi.VdxsConfig) == 32
    offs = [getattr(abi.VdxsConfig, n).offset for n, _ in abi.VdxsConfig._fields_]
    assert offs == [0, 4, 8, 12, 16, 20, 24]


def test_default_config_from_library(lib):
    c = abi.VdxsConfig()
    lib.vdxs_default_config(C.byref(c))
    assert c.as_dict() == dict(temperature=0.0, top_k=0, top_p=1.0, min_p=0.0, repeat_penalty=1.0,
                               repeat_window=64, seed=0)
    assert lib.vdxs_abi_version() == abi.ABI_VERSION


def test_null_arguments_are_rejected_without_a_gpu(lib):
    c = abi.default_config(temperature=1.0, top_k=4)
    rc = lib.vdxs_sample(None, C.byref(c), None, 0, 1, 10, 10, None, 1, None, None, None, None)
    assert rc == abi.E_INVALID_ARG
    assert b"NULL" in lib.vdxs_last_error(None)
    assert lib.vdxs_create(0, None) == abi.E_INVALID_ARG


def test_missing_library_fails_loudly(tmp_path):
    saved = _lib._lib
    _lib._lib = None
    try:
        with pytest.raises(ImportError):
            _lib.load(str(tmp_path / "nope.so"))
    finally:
        _lib._lib = saved


def test_product_never_imports_the_oracle():
    pkg = os.path.join(ROOT, "vindexllm_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cpp", ".h", ".cuh")):
                text = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in text and "from oracle" not in text and "vdx_oracle" not in text, f
