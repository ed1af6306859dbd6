"""The C-ABI library loads and exports every symbol include/gptb200.h declares
(no GPU needed), and argument errors come back as status codes."""

import ctypes
import pathlib
import re

from rig_b200 import _lib

HEADER = pathlib.Path(__file__).resolve().parent.parent / "include" / "gptb200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gptb200_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing


def test_python_binding_covers_header():
    assert set(declared_functions()) <= set(_lib.SIGNATURES)


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.gptb200_version().startswith(b"gptb200")
    assert lib.gptb200_status_string(0) == b"ok"
    assert b"shape" in lib.gptb200_status_string(2)


def test_argument_errors_are_status_codes():
    lib = _lib.load()
    # null pointers are rejected before anything touches a device
    assert lib.gptb200_rms_norm_fwd(None, None, None, None, 10, 64, None) == 1
    assert lib.gptb200_lce_fwd(None, None, None, 1, 8, 8, 8, None, None, None, None, None) == 1
    assert lib.gptb200_attention_bwd_workspace_size(0, 1, 1) == 0
    assert lib.gptb200_lce_fwd_workspace_size(131072, 50304) > 131072 * 197 * 8
    # scratch sizes are pure host arithmetic
    assert lib.gptb200_gemm_workspace_size(768, 768, 131072, _lib.EPI_F32) == 0
    assert lib.gptb200_gemm_workspace_size(768, 768, 64, _lib.EPI_F32_SPLITK) == 0
    assert lib.gptb200_embedding_bwd_workspace_size(131072, 768, 50304) >= 4 * 131072 * 4
    assert lib.gptb200_embedding_bwd(None, None, None, 8, 8, 8, None, None) == 1
    assert lib.gptb200_colsum(None, 8, 8, 1.0, None, None, None) == 1
