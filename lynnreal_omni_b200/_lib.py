"""ctypes binding of liblr_w8a8.so, the sm_100a C ABI declared in include/lr_w8a8.h.

The library is the only compute path: if it is missing or cannot be loaded the
ops raise instead of falling back to another implementation.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import torch

PACKAGE = Path(__file__).resolve().parent
LIBRARY = PACKAGE / "liblr_w8a8.so"
HEADER = PACKAGE.parent / "include" / "lr_w8a8.h"

LR_OK = 0
LR_ERR_INVALID_ARGUMENT = 1
LR_ERR_UNSUPPORTED = 2
LR_ERR_CUDA = 3

LR_EPI_NONE = 0
LR_EPI_GELU_TANH = 1
LR_EPI_GATED_RESIDUAL = 2

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float

# argument types of every entry point, in header order
SIGNATURES = {
    "lr_version": ([], _i32),
    "lr_last_error": ([], ctypes.c_char_p),
    "lr_device_status": ([ctypes.POINTER(ctypes.c_uint), _i32], _i32),
    "lr_set_arithmetic": ([_i32], _i32),
    "lr_get_arithmetic": ([ctypes.POINTER(ctypes.c_int)], _i32),
    "lr_quantize_rows": ([_p, _i64, _i64, _i64, _p, _p, _p], _i32),
    "lr_quantize_rows_arith": ([_p, _i64, _i64, _i64, _p, _p, _i32, _p], _i32),
    "lr_int8_epilogue": ([_p, _i64, _i64, _p, _p, _p, _p, _p], _i32),
    "lr_rms_adaln": ([_p, _p, _f32, _p, _i64, _i64, _p, _i64, _i64, _i64, _i32, _i32, _p, _p], _i32),
    "lr_rms_adaln_quant_int8": ([_p, _p, _f32, _p, _i64, _i64, _p, _i64, _i64, _i64, _i32, _i32,
                                 _p, _i32, _p, _p, _p, _p], _i32),
    "lr_gated_residual": ([_p, _p, _p, _i64, _i64, _p, _i64, _i64, _i64, _i32, _p, _p], _i32),
    "lr_swiglu": ([_p, _i64, _i64, _p, _p], _i32),
    "lr_swiglu_quant_int8": ([_p, _i64, _i64, _p, _p, _p], _i32),
    "lr_qk_norm_rope": ([_p, _p, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _f32,
                         _p, _p, _p], _i32),
    "lr_gather_rows": ([_p, _i64, _i64, _i64, _i64, _p, _i64, _p, _i64, _p], _i32),
    "lr_flash_restore": ([_p, _p, _p, _p, _i64, _i64, _i64, _i64, _f32, _p, _p], _i32),
    "lr_flash_nearest_anchor": ([_p, _i64, _p, _i64, _p, _i64, _p, _p], _i32),
    "lr_attention_bf16": ([_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _p, _i64, _p], _i32),
    "lr_int8_gemm": ([_p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _i32, _p, _i64, _p,
                      _i64, _i64, _p, _i64, _i32, _p, _i64, _p], _i32),
    "lr_int8_gemm_workspace_bytes": ([_i64, _i64, _i64], _i64),
    "lr_int8_gemm_ws": ([_p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _i32, _p, _i64, _p,
                         _i64, _i64, _p, _i64, _i32, _p, _i64, _p, _i64, _p], _i32),
    "lr_int8_gemm_noalloc": ([_p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _i32, _p, _i64, _p,
                              _i64, _i64, _p, _i64, _i32, _p, _i64, _p], _i32),
    "lr_int8_gemm_s32": ([_p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _p, _p], _i32),
    "lr_int8_gemm_rows_to": ([_p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _i32, _p, _i64, _p,
                              _i64, _i64, _p, _i64, _i32, _p, _i32, _i64, _i64, _p], _i32),
    "lr_gemm_test_wait": ([_i64, _i32], _i32),
    "lr_ipc_export": ([_p, _p, ctypes.POINTER(ctypes.c_int64)], _i32),
    "lr_ipc_import": ([_p, _i64, ctypes.POINTER(ctypes.c_void_p)], _i32),
    "lr_ipc_release": ([_p, _i64], _i32),
}

_lib = None


class LibraryError(RuntimeError):
    """The sm_100a library is missing or could not be loaded."""


def header_symbols() -> list[str]:
    """Names of the entry points declared in include/lr_w8a8.h."""
    text = HEADER.read_text()
    return re.findall(r"^(?:int|int64_t|const char\*)\s+(lr_\w+)\s*\(", text, flags=re.M)


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load the library once and declare every entry point's signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    target = Path(path) if path is not None else LIBRARY
    if not target.exists():
        raise LibraryError(f"{target} is missing; build it with `python -m lynnreal_omni_b200.build`")
    try:
        lib = ctypes.CDLL(str(target))
    except OSError as error:
        raise LibraryError(f"cannot load {target}: {error}") from error
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    if path is None:
        _lib = lib
    return lib


def check(status: int, what: str) -> None:
    """Raise the reference's exception type for a failed C-ABI call."""
    if status == LR_OK:
        return
    message = (load().lr_last_error() or b"").decode(errors="replace")
    if status in (LR_ERR_INVALID_ARGUMENT, LR_ERR_UNSUPPORTED):
        raise ValueError(f"{what}: {message}")
    raise RuntimeError(f"{what}: {message}")


def ptr(tensor: torch.Tensor | None) -> int | None:
    return None if tensor is None else tensor.data_ptr()


def stream_of(tensor: torch.Tensor) -> int:
    """The caller's current CUDA stream on the tensor's device (launch target)."""
    if tensor.device.type != "cuda":
        raise ValueError("the W8A8 ops run on CUDA tensors only")
    return torch.cuda.current_stream(tensor.device).cuda_stream


ARITHMETIC = {"reference_gpu": 1, "ieee": 0}
# per-call quantiser arithmetic only (lr_quantize_rows_arith): the reference's
# unfused PyTorch quantiser on a CUDA device
LR_ARITH_TORCH_CUDA = 2


def set_arithmetic(mode: str) -> None:
    """Arithmetic of the element-wise kernels' divisions and RMS reciprocal
    square roots on the current device: "reference_gpu" (default; as the
    reference's compiled Triton kernels) or "ieee" (as its PyTorch path and
    the CPU oracle)."""
    if mode not in ARITHMETIC:
        raise ValueError(f"arithmetic must be one of {sorted(ARITHMETIC)}, got {mode!r}")
    check(load().lr_set_arithmetic(ARITHMETIC[mode]), "set_arithmetic")


def arithmetic() -> str:
    """The current device's arithmetic mode (see set_arithmetic)."""
    value = ctypes.c_int(0)
    check(load().lr_get_arithmetic(ctypes.byref(value)), "arithmetic")
    return {v: k for k, v in ARITHMETIC.items()}[value.value]


def device_status(clear: bool = True) -> int:
    """Device status bits (1: adaLN index out of range, 2: GEMM wait timeout)."""
    bits = ctypes.c_uint(0)
    check(load().lr_device_status(ctypes.byref(bits), int(clear)), "device_status")
    return bits.value
