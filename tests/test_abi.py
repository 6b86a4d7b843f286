"""The C-ABI library: built, loadable, exports every symbol of include/gqa.h,
and rejects bad arguments with a status code (no GPU needed, no compute)."""
import ctypes
import os
import subprocess

import pytest


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.lib()
    declared = pkg.header_functions()
    assert len(declared) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", pkg.gqa.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [f for f in declared if f not in exported]
    assert not missing, f"declared but not exported: {missing}"
    for f in declared:
        assert hasattr(lib, f)
    # only the C ABI is exported
    extra = sorted(e for e in exported if not e.startswith("gqa_"))
    assert not extra, f"unexpected exports: {extra[:10]}"


def test_library_is_sm100a_only(pkg):
    out = subprocess.run(["cuobjdump", "--list-elf", pkg.gqa.LIB_PATH], capture_output=True,
                         text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    assert "sm_100a" in out.stdout


def test_version_and_error_string(pkg):
    assert b"sm_100a" in pkg.lib().gqa_version()
    assert isinstance(pkg.last_error(), str)


def test_null_arguments_are_rejected(pkg):
    lib = pkg.lib()
    assert lib.gqa_create(None, 0, None) == pkg.gqa.GQA_ERR_INVALID_ARG
    assert "null" in pkg.last_error()
    assert lib.gqa_layer_attention(None, None, None, None, 0, 1) == pkg.gqa.GQA_ERR_INVALID_ARG
    assert lib.gqa_decode_batched(None, None, 0, None, None, None, 0, None, 0, None, 0) \
        == pkg.gqa.GQA_ERR_INVALID_ARG
    assert lib.gqa_destroy(None) == 0


def test_unsupported_shapes_are_rejected_before_touching_the_device(pkg):
    lib = pkg.lib()
    h = ctypes.c_void_p()
    bad = pkg.gqa.Config(12, 2, 64, 4096, 1e6)  # head_dim 64 is built with 7 per KV head only
    assert lib.gqa_create(ctypes.byref(bad), 0, ctypes.byref(h)) == pkg.gqa.GQA_ERR_UNSUPPORTED
    bad = pkg.gqa.Config(14, 2, 128, 4096, 1e6)  # group 7 is built at head_dim 64 only
    assert lib.gqa_create(ctypes.byref(bad), 0, ctypes.byref(h)) == pkg.gqa.GQA_ERR_UNSUPPORTED
    bad = pkg.gqa.Config(12, 2, 128, 0, 1e6)
    assert lib.gqa_create(ctypes.byref(bad), 0, ctypes.byref(h)) == pkg.gqa.GQA_ERR_INVALID_ARG


def test_no_device_is_an_error_not_a_crash(pkg):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(pkg.GqaError):
        pkg.Context()


def test_package_has_no_cpu_fallback(pkg):
    src = open(pkg.gqa.__file__).read()
    assert "oracle" not in src.replace("# ", "")
    assert os.path.basename(pkg.gqa.LIB_PATH) == "libgqa_b200.so"
