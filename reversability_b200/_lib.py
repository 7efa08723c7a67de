"""ctypes binding of librevk.so (the C ABI declared in include/revk.h).

The library is loaded once, from this package directory. Every call passes
raw device pointers, element counts and the current CUDA stream; a non-zero
status becomes a RuntimeError carrying the library's own message. There is no
fallback: if the library is missing, every kernel entry point raises.
"""
from __future__ import annotations

import contextlib
import ctypes
import re
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "librevk.so"
HEADER = Path(__file__).resolve().parents[1] / "include" / "revk.h"

F32, BF16, F16 = 0, 1, 2
ERR_ALIGN = 2  # RK_ERR_ALIGN: a pointer or leading dimension breaks a vector/TMA alignment rule
ERR_UNSUPPORTED = 5  # RK_ERR_UNSUPPORTED: the shape or layout is outside what a kernel implements
DTYPE_CODE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i = ctypes.c_int
_f = ctypes.c_float

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "rk_abi_version": (_i, []),
    "rk_launch_count": (ctypes.c_ulonglong, []),
    "rk_status_string": (ctypes.c_char_p, [_i]),
    "rk_device_status_read": (_i, [ctypes.POINTER(ctypes.c_uint), _p]),
    "rk_rmsnorm_fwd": (_i, [_p, _i, _i64, _p, _p, _i, _i64, _p, _i64, _i64, _f, _p]),
    "rk_rmsnorm_bwd_workspace": (_i64, [_i64, _i64]),
    "rk_rmsnorm_bwd": (_i, [_p, _i, _i64, _p, _p, _p, _i, _i64, _p, _i, _i64, _p, _i, _p, _i64, _i64, _i64, _p]),
    "rk_rmsnorm_bwd_noalloc": (_i, [_p, _i, _i64, _p, _p, _p, _i, _i64, _p, _i, _i64, _p, _i, _i64, _i64, _p]),
    "rk_swiglu_fwd": (_i, [_p, _p, _i, _i64, _i64, _p]),
    "rk_swiglu_bwd": (_i, [_p, _p, _p, _i, _i64, _i64, _p]),
    "rk_reconstruct_midpoint": (_i, [_p, _p, _i, _f, _p, _i64, _p]),
    "rk_reconstruct_euler": (_i, [_p, _p, _i, _p, _i64, _p]),
    "rk_gemm_fprop": (_i, [_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _i64, _i, _i, _p]),
    "rk_gemm_dgrad": (_i, [_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _i64, _i, _i, _p]),
    "rk_gemm_wgrad_workspace": (_i64, [_i64, _i64, _i64]),
    "rk_gemm_fprop_swiglu": (_i, [_p, _i64, _p, _i64, _p, _i64, _p, _i64, _i64, _i64, _i64, _i, _p]),
    "rk_gemm_dgrad_swiglu": (_i, [_p, _i64, _p, _i64, _p, _i64, _p, _i64, _i64, _i64, _i64, _i, _p]),
    "rk_gemm_dgrad_dsum": (_i, [_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _i64, _i, _p, _i64, _p, _i64, _i64, _p]),
    "rk_gemm_fprop_reconstruct": (_i, [_p, _i64, _p, _i64, _p, _i64, _p, _i64, _f, _p, _i64, _i64, _i64, _i64, _i,
                                       _p]),
    "rk_gemm_fprop_reconstruct_norm": (_i, [_p, _i64, _p, _i64, _p, _i64, _p, _i64, _f, _p, _i64, _p, _i64, _p, _f,
                                            _p, _i64, _p, _i64, _i64, _i64, _i, _p]),
    "rk_gemm_wgrad": (_i, [_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _i64, _i, _i, _p, _i64, _p]),
    "rk_attn_fwd": (_i, [_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _i64, _i, _p]),
    "rk_attn_bwd": (_i, [_p, _i64, _p, _p, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i, _p]),
    "rk_attn_bwd_piece": (_i, [_i, _p, _i64, _p, _p, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i, _p]),
    "rk_clip_adamw_workspace": (_i64, []),
    "rk_clip_adamw_prepare": (_i, [_p, _i64, _f, _f, _f, _f, _p, _i64, _p, _p]),
    "rk_adamw_step": (_i, [_p, _p, _p, _p, _p, _i, _i64, _p, _f, _f, _f, _p]),
    "rk_embedding_fwd": (_i, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _p]),
    "rk_embedding_bwd_workspace": (_i64, [_i64, _i64]),
    "rk_embedding_bwd": (_i, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _i64, _p]),
    "rk_embedding_bwd_sort_bytes": (_i64, [_i64, _i64]),
    "rk_embedding_bwd_sort": (_i, [_p, _i64, _i64, _p, _i64, _p]),
    "rk_embedding_bwd_sorted_workspace": (_i64, [_i64, _i64]),
    "rk_embedding_bwd_sorted": (_i, [_p, _i64, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _i64, _p]),
    "rk_layer_workspace": (_i64, [_p, _i, _i]),
    "rk_layer_fwd_midpoint": (_i, [_p, _p, _p, _f, _p, _p, _i64, _p]),
    "rk_layer_fwd_euler": (_i, [_p, _p, _p, _p, _p, _p, _i64, _p]),
    "rk_layer_bwd_midpoint": (_i, [_p, _p, _p, _p, _p, _p, _p, _f, _p, _p, _p, _p, _i64, _p]),
    "rk_layer_bwd_euler": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p]),
    "rk_reconstruct_midpoint_sum": (_i, [_p, _p, _p, _i, _f, _p, _i64, _p]),
    "rk_cast_scale": (_i, [_p, _p, _i, _f, _i64, _p]),
    "rk_add_rmsnorm_fwd": (_i, [_p, _p, _i, _p, _p, _i, _p, _p, _i64, _i64, _f, _p]),
    "rk_rmsnorm_bwd_fused": (_i, [_p, _p, _p, _p, _i, _p, _p, _p, _i, _f, _p, _p, _i, _p, _i64, _i64, _i64, _p]),
    "rk_rmsnorm_dw_reduce": (_i, [_p, _i64, _i64, _p, _i, _p]),
    "rk_cross_entropy_fwd_bwd": (_i, [_p, _i64, _i64, _p, _i64, _f, _p, _p, _p, _i64, _i, _i, _p]),
    "rk_head_stats_width": (_i64, [_i64]),
    "rk_head_fprop": (_i, [_p, _i64, _p, _i64, _p, _p, _i64, _p, _p, _i64, _i64, _i64, _i, _p]),
    "rk_head_loss": (_i, [_p, _i64, _p, _p, _i64, _i64, _f, _p, _p, _p, _p, _i64, _i, _p]),
    "rk_head_dgrad": (_i, [_p, _i64, _p, _i64, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i, _i, _p]),
    "rk_head_dgrad_workspace": (_i64, [_i64, _i64, _i64]),
    "rk_head_dgrad_ws": (_i, [_p, _i64, _p, _i64, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i, _i, _p, _i64,
                              _p]),
    "rk_head_wgrad": (_i, [_p, _i64, _p, _i64, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i, _i, _p]),
}

_lock = threading.Lock()
_lib = None


class KernelLibraryMissing(RuntimeError):
    pass


class LayerDesc(ctypes.Structure):
    """rk_layer_desc of include/revk.h (pointers as integers)."""
    _fields_ = [("batch", _i64), ("length", _i64), ("d_model", _i64), ("n_heads", _i64), ("d_ff", _i64),
                ("mlp_tokens", _i64), ("dtype", _i), ("eps_attn", _f), ("eps_mlp", _f),
                ("attn_norm", _p), ("qkv", _p), ("proj", _p), ("mlp_norm", _p), ("up", _p), ("down", _p)]


class LayerGrads(ctypes.Structure):
    """rk_layer_grads of include/revk.h."""
    _fields_ = [("attn_norm", _p), ("qkv", _p), ("proj", _p), ("mlp_norm", _p), ("up", _p), ("down", _p)]


METHOD_MIDPOINT, METHOD_EULER = 0, 1


def header_symbols() -> list[str]:
    """Every entry point declared in include/revk.h."""
    text = HEADER.read_text()
    return re.findall(r"^RK_API\s+[\w\s\*]+?\b(rk_\w+)\s*\(", text, flags=re.M)


def lib():
    """Loads librevk.so on first use; raises KernelLibraryMissing if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise KernelLibraryMissing(
                f"{LIB_PATH.name} is not built; run `python -m reversability_b200.build` (no CPU fallback exists)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def launch_count() -> int:
    """Kernel launches issued by librevk so far in this process."""
    return int(lib().rk_launch_count())


def status_string(code: int) -> str:
    return lib().rk_status_string(code).decode()


def check(code: int, name: str) -> None:
    if code != 0:
        raise RuntimeError(f"{name} failed: status {code} ({status_string(code)})")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


_launch_override: list[int] = []  # stack of stream handles set by launch_on()


def stream_ptr(device: torch.device | None = None) -> int:
    """The stream library kernels are launched on: the current CUDA stream, or
    the innermost launch_on() stream."""
    if _launch_override:
        return _launch_override[-1]
    return torch.cuda.current_stream(device).cuda_stream


@contextlib.contextmanager
def launch_on(stream: "torch.cuda.Stream"):
    """Library kernels issued inside the block go to `stream` while PyTorch
    keeps allocating on the current stream. The caller orders `stream` after
    the current stream's work before the block and keeps every tensor the
    block touches alive until the current stream has waited for `stream`, so
    the allocator never hands that memory to other work too early."""
    _launch_override.append(stream.cuda_stream)
    try:
        yield
    finally:
        _launch_override.pop()


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODE[dtype]
    except KeyError:
        raise ValueError(f"dtype {dtype} is not supported by the CUDA kernels") from None


def device_status(device: torch.device | None = None) -> int:
    """Reads and clears the library's device status word (synchronises the stream)."""
    out = ctypes.c_uint(0)
    check(lib().rk_device_status_read(ctypes.byref(out), stream_ptr(device)), "rk_device_status_read")
    return out.value
