"""ctypes binding of the C ABI in ``include/femtovllm_b200.h``.

This is the binding a ctypes-based caller of ``libfemtovllm_b200.so`` uses;
the GPU parity tests go through it so the exact ``extern "C"`` entry points
are what gets checked.  Pointers are passed as integers (``tensor.data_ptr()``),
streams as the raw ``cudaStream_t`` (``torch.cuda.current_stream().cuda_stream``).
Loading the library needs no GPU; calling a compute entry point does.
"""

from __future__ import annotations

import ctypes
import re
from ctypes import c_char_p, c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

from femtovllm_b200 import LIB_PATH

HEADER = Path(__file__).resolve().parents[2] / "include" / "femtovllm_b200.h"

FVB_DTYPE_F32, FVB_DTYPE_BF16, FVB_DTYPE_F16 = 0, 1, 2
FVB_OK = 0
STATUS_NAMES = {
    0: "FVB_OK",
    1: "FVB_ERR_INVALID_ARGUMENT",
    2: "FVB_ERR_UNSUPPORTED",
    3: "FVB_ERR_MISALIGNED",
    4: "FVB_ERR_WORKSPACE_TOO_SMALL",
    5: "FVB_ERR_CUDA",
    6: "FVB_ERR_DEVICE_TIMEOUT",
    7: "FVB_ERR_BAD_PAGE",
    8: "FVB_ERR_BAD_SLOT",
    9: "FVB_ERR_NO_DEVICE_SUPPORT",
}

_SIGNATURES = {
    "fvb_status_string": (c_char_p, [c_int]),
    "fvb_last_cuda_error": (c_int, []),
    "fvb_kv_len_per_page": (c_int, []),
    "fvb_dim_head": (c_int, []),
    "fvb_max_kv_len": (c_int, []),
    "fvb_read_device_error": (c_int, [ctypes.POINTER(c_int), ctypes.POINTER(c_int), c_void_p]),
    "fvb_check_bounded_wait": (c_int, [c_int, c_void_p]),
    "fvb_store_kvcache": (
        c_int,
        [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_int, c_int, c_int,
         c_int, c_void_p],
    ),
    "fvb_build_slot_mapping": (
        c_int, [c_void_p, c_int64, c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p]
    ),
    "fvb_build_varlen_metadata": (
        c_int,
        [c_void_p, c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int, c_int64, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p],
    ),
    "fvb_qk_norm_rope_store": (
        c_int,
        [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p,
         c_float, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_void_p, c_void_p,
         c_void_p, c_int64, c_int, c_int, c_void_p],
    ),
    "fvb_sample_workspace_size": (c_size_t, [c_int, c_int64]),
    "fvb_sample_tokens": (
        c_int,
        [c_void_p, c_int64, c_int, c_int64, c_int, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
         c_void_p, c_void_p, c_size_t, c_void_p],
    ),
    "fvb_paged_attention_decode_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "fvb_paged_attention_decode": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_int, c_void_p, c_int,
         c_void_p, c_int, c_int, c_void_p, c_size_t, c_void_p],
    ),
    "fvb_paged_attention_decode_strided": (
        c_int,
        [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int, c_int, c_int,
         c_int, c_int, c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_size_t, c_void_p],
    ),
    "fvb_paged_attention_prefill_strided": (
        c_int,
        [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int, c_int, c_int,
         c_int, c_int, c_int64, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_size_t,
         c_void_p],
    ),
    "fvb_paged_attention_prefill_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int, c_int64, c_int]),
    "fvb_paged_attention_prefill": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_int, c_int64, c_void_p,
         c_int, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_size_t, c_void_p],
    ),
}

_lib = None


def header_symbols() -> list[str]:
    """Every ``fvb_*`` function declared in include/femtovllm_b200.h."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"FVB_API\s+[\w\s\*]*?\b(fvb_\w+)\s*\(", text)))


def load(path: str | Path | None = None) -> ctypes.CDLL:
    """Load libfemtovllm_b200.so (once) and attach the ctypes signatures."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    lib = ctypes.CDLL(str(path or LIB_PATH))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


class FvbError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {STATUS_NAMES.get(status, status)}")


def check(status: int, what: str) -> None:
    if status != FVB_OK:
        if status == 5 and _lib is not None:  # FVB_ERR_CUDA: name the runtime error
            raise FvbError(status, f"{what} (cudaError {_lib.fvb_last_cuda_error()})")
        raise FvbError(status, what)


def dtype_code(dtype) -> int:
    import torch

    return {torch.float32: FVB_DTYPE_F32, torch.bfloat16: FVB_DTYPE_BF16, torch.float16: FVB_DTYPE_F16}[dtype]
