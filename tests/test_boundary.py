"""The C-ABI boundary: libkvcuda.so builds for sm_100a, loads, and exports every
entry point include/kvcuda.h declares; without a GPU it fails loudly (no CPU
fallback).  No compute calls are made here."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kvcuda.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b((?:kvcu|kvcache)_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def built_lib():
    import importlib.util

    spec = importlib.util.spec_from_file_location("kvbuild", os.path.join(ROOT, "mobile-moe.zig_b200", "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build()


def test_library_exports_every_declared_symbol(built_lib):
    out = subprocess.run(["nm", "-D", "--defined-only", built_lib], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r" T ((?:kvcu|kvcache)_[a-z0-9_]+)", out))
    declared = _declared()
    assert len(declared) > 50
    missing = [s for s in declared if s not in exported]
    assert not missing, missing


def test_binding_covers_the_header(built_lib):
    import kvcu

    assert sorted(kvcu.declared_symbols()) == _declared()
    kvcu.lib()  # loads and binds every signature


def test_build_targets_sm100a_only():
    src = open(os.path.join(ROOT, "mobile-moe.zig_b200", "build.py")).read()
    # one -gencode, sm_100a: the product ships no generic or older-arch path
    assert src.count("-gencode") == 1 and "arch=compute_100a,code=sm_100a" in src


def test_no_device_fails_loudly(built_lib):
    import torch

    import kvcu

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert kvcu.device_count() == 0
    with pytest.raises(kvcu.KVCudaError) as e:
        kvcu.init(0)
    assert e.value.name == "NoDevice"
    with pytest.raises(kvcu.KVCudaError):
        kvcu.KVCache(1, 512, 64, 64)
