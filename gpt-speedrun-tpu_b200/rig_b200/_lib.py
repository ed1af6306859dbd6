"""ctypes binding of libgptb200.so, the C ABI declared in include/gptb200.h.

The shared object is built in-tree by ``gpt-speedrun-tpu_b200/build.py``. There
is no fallback: if the library is missing, importing a compute entry point
raises, so a GPU run can never silently take a CPU or PyTorch path.
"""

from __future__ import annotations

import ctypes
import os
import pathlib

_HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = _HERE / "libgptb200.so"

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_f32 = ctypes.c_float
c_vp = ctypes.c_void_p
c_size = ctypes.c_size_t


class Epilogue(ctypes.Structure):
    _fields_ = [
        ("kind", c_int),
        ("accumulate", c_int),
        ("alpha", c_f32),
        ("bias", c_vp),
        ("residual", c_vp),
        ("ld_residual", c_i64),
        ("aux", c_vp),
        ("ld_aux", c_i64),
        ("rope_cos", c_vp),
        ("rope_sin", c_vp),
        ("rope_seq", c_i64),
        ("rope_cols", c_i64),
        ("row_range", c_vp),
        ("range_dim", c_int),
        ("workspace", c_vp),
    ]


class TensorGroup(ctypes.Structure):
    _fields_ = [
        ("offset", c_i64),
        ("size", c_i64),
        ("lr_mult", c_f32),
        ("eps_mult", c_f32),
        ("wd_mult", c_f32),
        ("decay", ctypes.c_int32),
    ]


class AdamWConfig(ctypes.Structure):
    _fields_ = [
        ("learning_rate", c_f32),
        ("horizon_lr_scale", c_f32),
        ("min_lr_ratio", c_f32),
        ("warmup_steps", ctypes.c_int32),
        ("total_steps", ctypes.c_int32),
        ("beta1", c_f32),
        ("beta2", c_f32),
        ("eps", c_f32),
        ("eps_horizon_scale", c_f32),
        ("weight_decay", c_f32),
        ("wd_horizon_scale", c_f32),
        ("grad_clip", c_f32),
        ("grad_scale", c_f32),
    ]


EPI_BF16 = 0
EPI_BIAS_GELU = 1
EPI_DGELU = 2
EPI_F32 = 3
EPI_F32_ATOMIC = 4
EPI_BIAS_ROPE = 5
EPI_F32_SPLITK = 6

DEVERR_GEMM = 1
DEVERR_ATTENTION = 2
DEVERR_TOKEN_RANGE = 4
DEVERR_NONFINITE = 8

# name -> (restype, argtypes). Mirrors include/gptb200.h one to one.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "gptb200_version": (ctypes.c_char_p, []),
    "gptb200_status_string": (ctypes.c_char_p, [c_int]),
    "gptb200_device_error": (c_int, [c_int]),
    "gptb200_device_error_flags": (c_int, [c_int]),
    "gptb200_launch_count": (ctypes.c_uint64, []),
    "gptb200_gemm": (
        c_int,
        [c_vp, c_int, c_i64, c_vp, c_int, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64,
         ctypes.POINTER(Epilogue), c_vp],
    ),
    "gptb200_rms_norm_fwd": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_vp]),
    "gptb200_gemm_workspace_size": (c_size, [c_i64, c_i64, c_i64, c_int]),
    "gptb200_rms_norm_bwd_workspace_size": (c_size, [c_i64, c_i64]),
    "gptb200_rms_norm_bwd": (
        c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_f32, c_i64, c_i64, c_vp, c_vp]),
    "gptb200_embedding_fwd": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp]),
    "gptb200_embedding_bwd_workspace_size": (c_size, [c_i64, c_i64, c_i64]),
    "gptb200_embedding_bwd": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "gptb200_rope_tables": (c_int, [c_vp, c_vp, c_i64, c_i64, c_vp]),
    "gptb200_document_segments": (c_int, [c_vp, c_i64, c_i64, ctypes.c_int32, c_vp, c_vp]),
    "gptb200_rope_apply": (
        c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_int, c_vp]),
    "gptb200_attention_fwd": (
        c_int,
        [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64, c_vp,
         c_i64, c_i64, c_i64, c_i64, c_f32, c_vp, c_vp],
    ),
    "gptb200_attention_bwd_workspace_size": (c_size, [c_i64, c_i64, c_i64]),
    "gptb200_attention_bwd": (
        c_int,
        [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp,
         c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_f32, c_vp, c_vp, c_vp, c_vp, c_vp],
    ),
    "gptb200_lce_fwd_workspace_size": (c_size, [c_i64, c_i64]),
    "gptb200_lce_fwd": (
        c_int,
        [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp],
    ),
    "gptb200_lce_fwd_noalloc": (
        c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp]),
    "gptb200_lce_bwd_workspace_size": (c_size, [c_i64, c_i64]),
    "gptb200_lce_bwd": (
        c_int,
        [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp],
    ),
    "gptb200_colsum_workspace_size": (c_size, [c_i64, c_i64]),
    "gptb200_colsum": (c_int, [c_vp, c_i64, c_i64, c_f32, c_vp, c_vp, c_vp]),
    "gptb200_moe_rows": (c_size, [c_i64, ctypes.c_int32, ctypes.c_int32]),
    "gptb200_moe_dispatch_workspace_size": (c_size, [c_i64, ctypes.c_int32, ctypes.c_int32]),
    "gptb200_moe_route": (
        c_int, [c_vp, c_vp, c_i64, c_i64, ctypes.c_int32, ctypes.c_int32, c_vp, c_vp, c_vp, c_vp,
                c_vp]),
    "gptb200_moe_dispatch": (
        c_int, [c_vp, c_i64, ctypes.c_int32, ctypes.c_int32, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp,
                c_vp, c_vp, c_vp]),
    "gptb200_moe_combine": (
        c_int, [c_vp, c_vp, c_vp, c_vp, c_f32, c_i64, c_i64, ctypes.c_int32, c_vp, c_vp]),
    "gptb200_moe_combine_bwd": (
        c_int, [c_vp, c_f32, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, ctypes.c_int32, c_vp,
                c_vp, c_vp]),
    "gptb200_moe_route_bwd": (
        c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64,
                ctypes.c_int32, ctypes.c_int32, c_vp, c_vp, c_vp]),
    "gptb200_moe_segment_colsum": (c_int, [c_vp, c_vp, ctypes.c_int32, c_i64, c_vp, c_vp]),
    "gptb200_moe_finalize": (
        c_int, [c_vp, ctypes.c_int32, ctypes.c_int32, c_i64, ctypes.c_int32, c_f32, c_f32, c_vp,
                c_vp, c_vp, ctypes.c_int32, c_vp, c_vp]),
    "gptb200_masked_loss_sum": (c_int, [c_vp, c_vp, c_i64, c_vp, c_vp]),
    "gptb200_adamw_workspace_size": (c_size, [c_i64]),
    "gptb200_adamw_step": (
        c_int,
        [c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, ctypes.c_int32, ctypes.POINTER(AdamWConfig),
         c_vp, c_vp, c_vp, c_vp, c_vp, c_vp],
    ),
    "gptb200_adamw_begin": (c_int, [ctypes.POINTER(AdamWConfig), c_vp, c_vp, c_vp]),
    "gptb200_adamw_update_range": (
        c_int,
        [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_vp, ctypes.c_int32, ctypes.POINTER(AdamWConfig),
         ctypes.c_int32, c_vp, c_vp, c_vp],
    ),
    "gptb200_adamw_end": (
        c_int, [ctypes.c_int32, ctypes.POINTER(AdamWConfig), c_vp, c_vp, c_vp, c_vp, c_vp]),
    "gptb200_cast_bf16": (c_int, [c_vp, c_vp, c_i64, c_vp]),
    "gptb200_mix_uint64": (ctypes.c_uint64, [ctypes.c_uint64]),
    "gptb200_permute_bounded": (
        ctypes.c_uint64, [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64]),
    "gptb200_epoch_windows": (
        c_int,
        [ctypes.POINTER(c_vp), c_vp, c_i64, c_int, c_vp, c_i64, ctypes.c_uint64, c_i64, c_i64,
         c_i64, c_i64, c_vp],
    ),
}


class GptB200Error(RuntimeError):
    """A libgptb200 entry point returned a non-zero status."""


_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads libgptb200.so once and binds every exported signature."""

    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python gpt-speedrun-tpu_b200/build.py` "
            "(there is no CPU or PyTorch fallback for the rig_b200 kernels)"
        )
    lib = ctypes.CDLL(os.fspath(LIB_PATH), mode=ctypes.RTLD_GLOBAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = load().gptb200_status_string(status).decode()
        raise GptB200Error(f"{what} failed with status {status}: {msg}")


def call(name: str, *args) -> int:
    """Calls an entry point and raises GptB200Error on a non-zero status."""

    status = getattr(load(), name)(*args)
    check(status, name)
    return status
