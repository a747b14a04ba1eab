"""CPU: the C-ABI library loads and exports every entry point include/g4b200.h declares.

No compute runs here (this container has no GPU); argument checks that need no context do.
"""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from g4b200 import _abi

HEADER = Path(__file__).resolve().parent.parent / "include" / "g4b200.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(g4_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_reference_ops():
    names = declared_symbols()
    for op in ("g4_sliding_project_qkv", "g4_sliding_attention", "g4_sliding_attention_output",
               "g4_decoder_feedforward"):
        assert op in names


def test_library_exports_every_declared_symbol():
    lib = _abi.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_abi.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (g4_[a-z0-9_]+)$", out, flags=re.M))
    assert set(declared_symbols()) <= exported, set(declared_symbols()) - exported


def test_library_is_built_for_sm100a_only():
    """The build compiles every source for sm_100a and nothing else (no PTX to JIT elsewhere)."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("g4_build", HEADER.parent.parent / "moa-workspace_b200" / "build.py")
    build = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(build)
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_status_strings():
    lib = _abi.lib()
    assert lib.g4_status_string(0) == b"ok"
    assert lib.g4_status_string(-2) == b"misaligned pointer"
    assert lib.g4_status_string(12345) == b"unknown status"


def test_null_context_is_rejected():
    lib = _abi.lib()
    assert lib.g4_ctx_destroy(None) == _abi.G4_ERR_INVALID_ARGUMENT
    assert lib.g4_ctx_check(None, None, None) == _abi.G4_ERR_INVALID_ARGUMENT
    assert lib.g4_sliding_attention_output(None, None, None, None, None, None, None) == _abi.G4_ERR_INVALID_ARGUMENT
    assert lib.g4_ctx_create(0, None) == _abi.G4_ERR_INVALID_ARGUMENT


def test_ctx_create_without_gpu_fails_cleanly():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    handle = ctypes.c_void_p()
    st = _abi.lib().g4_ctx_create(0, ctypes.byref(handle))
    assert st != _abi.G4_OK and not handle
