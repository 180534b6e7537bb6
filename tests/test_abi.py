"""CPU tests of the C-ABI boundary: the library builds, loads without a GPU
and exports every entry point the public headers declare; compute calls
fail loudly (no CPU fallback) when no sm_100 device is present."""
import ctypes as C
import re
from pathlib import Path

import pytest

import moe_b200
from conftest import REPO, gpu_available

HEADERS = sorted((REPO / "include").glob("*.h"))


def declared_functions():
    names = set()
    for h in HEADERS:
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        text = re.sub(r"#[^\n]*", "", text)
        # a declaration: <type> name(args);  (skip typedef'd function pointers)
        for m in re.finditer(r"\b([A-Za-z_]\w*)\s*\([^;{]*\)\s*;", text):
            name = m.group(1)
            if name in {"sizeof", "if", "for", "while", "return"}:
                continue
            names.add(name)
    return names


def test_headers_declare_entry_points():
    names = declared_functions()
    assert {"moe_b200_forward", "moe_b200_forward_device", "moe_b200_weights_upload",
            "moe_forward", "moe_b200_invalidate"} <= names


def test_library_exports_every_declared_symbol():
    lib = moe_b200.lib()
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_version_and_strerror():
    assert "sm_100a" in moe_b200.version()
    lib = moe_b200.lib()
    for code in (0, -1, -2, -3, -4, -5, -6, -7):
        assert lib.moe_b200_strerror(code)


@pytest.mark.skipif(gpu_available(), reason="checks the no-GPU failure mode")
def test_no_gpu_fails_loudly():
    with pytest.raises(moe_b200.MoEError) as ei:
        moe_b200.init(0)
    assert ei.value.status in (moe_b200.E_NODEV, moe_b200.E_CUDA)


def test_built_for_sm100a_only():
    log = (REPO / "llm.c_b200" / "build.log")
    if not log.exists():
        pytest.skip("build log absent")
    text = log.read_text()
    assert "sm_100a" in text and "sm_90" not in text


def test_loading_library_before_torch_keeps_torch_importable():
    # the library resolves NCCL only when an expert-parallel group is made,
    # so loading it first must not pin an NCCL that torch cannot use
    import subprocess
    import sys
    code = ("import sys; sys.path.insert(0, 'llm.c_b200'); import moe_b200; "
            "moe_b200.lib(); import torch; print(torch.__version__)")
    subprocess.run([sys.executable, "-c", code], cwd=str(REPO), check=True, timeout=600)
