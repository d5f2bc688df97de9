"""ctypes binding of the C ABI in ``include/tropnn_b200.h``.

The reference's only foreign-function precedent for this path is the Zig CPU backend,
bound with ctypes through raw ``data_ptr()`` values and integer sizes
(backends/zig_runtime.py:75-164, backends/tropical_zig.py:35-107). This module binds the
sm_100a kernel library the same way. There is no fallback: if the library is missing
or cannot be loaded, every b200 op raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libtropnn_b200.so"
ABI_VERSION = 20

# tropnn_b200_dtype
F32, F16, BF16, U8, I16, I64 = 0, 1, 2, 3, 4, 5
# tropnn_b200_surrogate
SURROGATES = {"fast_sigmoid_odd": 0, "izhikevich": 1}

# tropnn_b200_status
OK = 0
ERR_INVALID = -1
ERR_DTYPE = -2
ERR_DEVICE = -3
ERR_LAUNCH = -4
ERR_WORKSPACE = -5
ERR_TIMEOUT = -6

_FLOAT_DTYPES = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
_INDEX_DTYPES = {torch.uint8: U8, torch.int16: I16, torch.int64: I64}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes), in the order of include/tropnn_b200.h.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "tropnn_b200_last_error": (ctypes.c_char_p, []),
    "tropnn_b200_abi_version": (_i32, []),
    "tropnn_b200_kernel_launches": (ctypes.c_ulonglong, []),
    "tropnn_b200_check_device": (_i32, [_i32]),
    "tropnn_b200_bucket_sort": (_i32, [_p, _i32, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "tropnn_b200_segment_rowsum": (
        _i32,
        [_p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _f32, _p, _p, _p, _f32, _f32, _p, _i32, _p, _p],
    ),
    "tropnn_b200_segment_rowsum_half": (
        _i32, [_p, _i32, _i64, _i64, _i64, _i64, _i64, _p, _p, _f32, _p, _p, _i32, _p]
    ),
    "tropnn_b200_pairwise_lut_grad": (_i32, [_p, _i64, _i64, _p, _i64, _i64, _f32, _p, _i32, _p]),
    "tropnn_b200_pairwise_lut_grad_peer_floats": (_i64, [_i64, _i64, _i64]),
    "tropnn_b200_pairwise_lut_grad_allreduce": (
        _i32,
        [_p, _i64, _i64, _p, _i64, _i64, _f32, _p, _i32, _p, _i32, _i32, _i64, _i32, _p],
    ),
    "tropnn_b200_pairwise_forward": (
        _i32,
        [_p, _i64, _i64, _p, _p, _i32, _i64, _i64, _p, _i32, _i64, _f32, _p, _p, _p, _p],
    ),
    "tropnn_b200_pairwise_anchor_index": (_i32, [_p, _i64, _i64, _i64, _p, _p, _p]),
    "tropnn_b200_pairwise_ste_backward": (
        _i32,
        [_p, _i64, _i64, _f32, _p, _p, _p, _i64, _i64, _i64, _p, _i32, _i32, _i32, _p, _p, _p, _p, _p, _p],
    ),
    "tropnn_b200_pairwise_threshold_grad_workspace_size": (_sz, [_i64, _i64, _i64]),
    "tropnn_b200_pairwise_threshold_grad": (_i32, [_p, _p, _i64, _i64, _i64, _i32, _p, _i32, _p, _sz, _p]),
    "tropnn_b200_pairwise_backward_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i32]),
    "tropnn_b200_pairwise_backward": (
        _i32,
        [_p, _i64, _i64, _f32, _p, _p, _p, _i64, _i64, _i64, _p, _i32, _i32, _i32, _p, _p, _i32, _p, _p, _sz, _p],
    ),
    "tropnn_b200_pairwise_backward_noalloc": (
        _i32,
        [_p, _i64, _i64, _f32, _p, _p, _p, _i64, _i64, _i64, _p, _i32, _i32, _i32, _p, _p, _i32, _p, _p],
    ),
    "tropnn_b200_trop_route_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i32, _i32]),
    "tropnn_b200_trop_route": (
        _i32, [_p, _i32, _i64, _i64, _p, _p, _i32, _i32, _i64, _i64, _p, _p, _p, _i32, _p, _p, _sz, _p]
    ),
    "tropnn_b200_trop_hidden_workspace_size": (_sz, [_i64, _i64, _i64, _i64]),
    "tropnn_b200_trop_hidden": (
        _i32,
        [_p, _i32, _i64, _i64, _p, _p, _i32, _i64, _i64, _p, _p, _i32, _p, _f32, _i32, _p, _p, _p, _sz, _p],
    ),
    "tropnn_b200_trop_code_transpose": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p]),
    "tropnn_b200_trop_proj_workspace_size": (_sz, [_i64, _i64, _i64]),
    "tropnn_b200_trop_proj": (_i32, [_p, _i64, _i64, _p, _i32, _i64, _p, _p, _sz, _p]),
    "tropnn_b200_trop_proj_wgrad_workspace_size": (_sz, [_i64, _i64, _i64]),
    "tropnn_b200_trop_proj_wgrad": (_i32, [_p, _i64, _i64, _p, _i32, _i64, _p, _p, _sz, _p]),
    "tropnn_b200_gemm_tf32x3_workspace_size": (_sz, [_i64, _i64, _i64]),
    "tropnn_b200_gemm_tf32x3": (_i32, [_p, _i64, _p, _i64, _i64, _i64, _i64, _p, _p, _i64, _p, _sz, _p]),
    "tropnn_b200_transpose_f32": (_i32, [_p, _i64, _i64, _i64, _p, _i64, _p]),
    "tropnn_b200_colsum_f32": (_i32, [_p, _i64, _i64, _i64, _p, _p]),
    "tropnn_b200_split_half": (_i32, [_p, _i64, _i64, _i32, _p, _p, _p]),
    "tropnn_b200_split_transpose_half": (_i32, [_p, _i64, _i64, _i32, _p, _p, _p, _p]),
    "tropnn_b200_absmax_f32": (_i32, [_p, _i64, _p, _p]),
    "tropnn_b200_linear_f32out": (_i32, [_p, _i64, _i64, _p, _i64, _i64, _i32, _p, _p, _p]),
    "tropnn_b200_peer_buffer_create": (_i32, [_i64, ctypes.POINTER(_p), _p]),
    "tropnn_b200_peer_buffer_open": (_i32, [_p, ctypes.POINTER(_p)]),
    "tropnn_b200_peer_buffer_close": (_i32, [_p]),
    "tropnn_b200_peer_buffer_destroy": (_i32, [_p]),
    "tropnn_b200_peer_allreduce_f32": (_i32, [_p, _i32, _i32, _i64, _p, _p, _i32, _i32, _p]),
    "tropnn_b200_device_error": (_i32, [ctypes.POINTER(ctypes.c_int)]),
    "tropnn_b200_trop_gm": (_i32, [_p, _i64, _i64, _p, _i32, _i64, _i64, _p, _p, _p, _f32, _p, _p, _p]),
    "tropnn_b200_trop_router_term": (_i32, [_p, _i64, _i64, _p, _i32, _i64, _i64, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "tropnn_b200_trop_param_grad": (_i32, [_i32, _p, _i64, _i64, _i32, _i64, _i64, _p, _p, _p, _f32, _p, _p, _p, _p]),
    "tropnn_b200_transpose_to_half": (_i32, [_p, _i32, _i64, _i64, _i32, _p, _p, _p]),
    "tropnn_b200_linear_dgrad_workspace_size": (_sz, [_i64, _i64, _i64]),
    "tropnn_b200_linear_dgrad": (_i32, [_p, _i64, _i64, _p, _i64, _p, _p, _sz, _p]),
    "tropnn_b200_linear_wgrad": (_i32, [_p, _i64, _i64, _p, _p, _i64, _i32, _p, _p, _p]),
    "tropnn_b200_tf32_split": (_i32, [_p, _i64, _p, _p, _p]),
    "tropnn_b200_trop_param_grad_rows": (
        _i32, [_p, _p, _i64, _i64, _i32, _i64, _i64, _p, _p, _i32, _p, _p, _f32, _p, _p, _p, _p, _p]
    ),
    "tropnn_b200_trop_backward_rows": (
        _i32,
        [_p, _i64, _i64, _p, _p, _i32, _i64, _i64, _p, _p, _i32, _p, _f32, _i32, _p, _p, _p, _p, _p],
    ),
    "tropnn_b200_trop_backward_workspace_size": (_sz, [_i64, _i64, _i64, _i32]),
    "tropnn_b200_trop_backward": (
        _i32,
        [_p, _p, _i64, _i64, _p, _p, _i32, _i64, _i64, _p, _p, _i32, _p, _f32, _i32, _p, _p, _p, _p, _p, _sz, _p],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class B200Unavailable(RuntimeError):
    """The sm_100a kernel library is missing or cannot run here."""


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Loads (once) the kernel library and declares every exported signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        lib_path = Path(path or os.environ.get("TROPNN_B200_LIB") or LIB_PATH)
        if not lib_path.exists():
            raise B200Unavailable(
                f"backend='b200' kernel library not found at {lib_path}; build it with "
                "`python -m tropnn_b200.build` (needs nvcc with sm_100a support)"
            )
        lib = ctypes.CDLL(str(lib_path))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        version = lib.tropnn_b200_abi_version()
        if version != ABI_VERSION:
            raise B200Unavailable(f"kernel library ABI {version} does not match the Python binding ABI {ABI_VERSION}")
        if path is None:
            _lib = lib
        return lib


def last_error() -> str:
    return load().tropnn_b200_last_error().decode(errors="replace")


def check(status: int, what: str) -> None:
    """Raises the reference's exception type for a failing status."""
    if status == OK:
        return
    message = f"{what}: {last_error()}"
    if status == ERR_INVALID:
        raise ValueError(message)
    if status == ERR_DTYPE:
        raise TypeError(message)
    raise RuntimeError(message)


def float_code(dtype: torch.dtype) -> int:
    try:
        return _FLOAT_DTYPES[dtype]
    except KeyError:
        raise TypeError(f"backend='b200' supports float32/float16/bfloat16 parameters, got {dtype}") from None


def index_code(dtype: torch.dtype) -> int:
    try:
        return _INDEX_DTYPES[dtype]
    except KeyError:
        raise TypeError(f"backend='b200' route indices must be uint8/int16/int64, got {dtype}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream
