"""ctypes binding of ``libfpv2_b200.so`` (the C ABI declared in include/fpv2_b200.h).

The library is the only compute path: when it is missing, or a tensor is not a
CUDA tensor, the operators raise instead of falling back to anything else.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

# FPV2_LIBRARY selects another build of the library (e.g. libfpv2_b200_debug.so,
# whose kernels report clamped list entries in the device status word).
LIB_PATH = Path(os.environ.get("FPV2_LIBRARY") or
                Path(__file__).resolve().parent / "_lib" / "libfpv2_b200.so")
STATUS_BAD_LIST = 8   # device status bit of the debug build's list bounds reports

F16, BF16, F32 = 0, 1, 2
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_DEVICE_TIMEOUT = 4
ATTN_WORKSPACE_BYTES = 16

_DTYPE_CODES = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32}

# Every exported entry point with its ctypes signature.
_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "fpv2_version": (ctypes.c_int, []),
    "fpv2_launch_count": (ctypes.c_int64, []),
    "fpv2_last_error": (ctypes.c_char_p, []),
    "fpv2_device_supported": (ctypes.c_int, [ctypes.c_int]),
    "fpv2_device_status": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int32)]),
    "fpv2_set_wait_budget_ms": (ctypes.c_int, [ctypes.c_double]),
    "fpv2_pool_blocks": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p],
    ),
    "fpv2_block_select": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_float, ctypes.c_int32, ctypes.c_int32, ctypes.c_float,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
         ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p],
    ),
    "fpv2_select_workspace_bytes": (
        ctypes.c_int64,
        [ctypes.c_int, ctypes.c_int, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32],
    ),
    "fpv2_compact_block_indices": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "fpv2_index_stage": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_float, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_float, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int,
         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p],
    ),
    "fpv2_sparse_attention": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
         ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
         ctypes.c_int, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_float,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
         ctypes.c_int64, ctypes.c_void_p],
    ),
    "fpv2_attention_workspace_bytes": (
        ctypes.c_int64,
        [ctypes.c_int, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int, ctypes.c_int32],
    ),
    "fpv2_sparse_attention_multicast": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
         ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
         ctypes.c_int, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_float,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p],
    ),
    "fpv2_sparse_attention_paged": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_float, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
         ctypes.c_void_p],
    ),
    "fpv2_pool_pages": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int,
         ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p],
    ),
    "fpv2_sparse_attention_noalloc": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
         ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
         ctypes.c_int, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_float,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "fpv2_fast_path_mask": (
        ctypes.c_int,
        [ctypes.c_int, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32],
    ),
    "fpv2_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_double, ctypes.c_void_p]),
}

EXPORTED_SYMBOLS = tuple(_SIGNATURES)

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class FPV2Error(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"fpv2 error {code}: {message}")
        self.code = code


def lib() -> ctypes.CDLL:
    """Load the shared library once and bind every signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built: run `python flashprefillv2-mlx_b200/build.py` "
                    "(the FPV2 operators have no fallback implementation)"
                )
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (restype, argtypes) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = handle
    return _lib


def check(rc: int) -> None:
    if rc != OK:
        msg = lib().fpv2_last_error().decode("utf-8", "replace")
        raise FPV2Error(rc, msg)


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError as error:
        raise ValueError(f"unsupported dtype {dtype}") from error


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> None:
    """FPV2 operators run only through the CUDA library: no host fallback."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError(
                "FPV2 B200 operators take CUDA tensors; there is no CPU implementation"
            )
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must be on the same CUDA device")


def launch_count() -> int:
    """Kernels the library has launched in this process so far (``fpv2_launch_count``)."""
    return int(lib().fpv2_launch_count())


def device_status(device: torch.device | int | None = None, clear: bool = True) -> int:
    """Synchronise the current stream and read (and clear) the device status word."""
    out = ctypes.c_int32(0)
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        stream = torch.cuda.current_stream().cuda_stream
        check(lib().fpv2_device_status(stream, 1 if clear else 0, ctypes.byref(out)))
    return int(out.value)


def attention_workspace(q: torch.Tensor, kv_heads: int, padded_k_len: int, block_k: int,
                        tile_q: int, pooled_dtype: torch.dtype, mean_correction: bool) -> torch.Tensor:
    """Device workspace for one attention call, sized by the library so that long
    work items can be split over the GPU (``fpv2_attention_workspace_bytes``)."""
    nbytes = lib().fpv2_attention_workspace_bytes(
        dtype_code(q.dtype), q.shape[0], kv_heads, q.shape[1], padded_k_len, q.shape[2], block_k,
        tile_q, dtype_code(pooled_dtype), 1 if mean_correction else 0)
    return torch.empty((max(int(nbytes), ATTN_WORKSPACE_BYTES) + 3) // 4, dtype=torch.int32,
                       device=q.device)


def select_workspace(q: torch.Tensor, pooled_dtype: torch.dtype, kv_heads: int, num_blocks: int,
                     head_dim: int) -> torch.Tensor | None:
    """Device workspace that lets the selection score float32 pooled keys on the
    tensor cores (``fpv2_select_workspace_bytes``); None when none is needed."""
    nbytes = int(lib().fpv2_select_workspace_bytes(
        dtype_code(q.dtype), dtype_code(pooled_dtype), kv_heads, num_blocks, head_dim))
    if nbytes <= 0:
        return None
    return torch.empty((nbytes + 3) // 4, dtype=torch.int32, device=q.device)


def workspace_args(ws: torch.Tensor | None) -> tuple[int | None, int]:
    return (None, 0) if ws is None else (ws.data_ptr(), ws.numel() * 4)


def set_wait_budget_ms(milliseconds: float) -> None:
    check(lib().fpv2_set_wait_budget_ms(float(milliseconds)))


def fast_path_mask(dtype: torch.dtype, q_heads: int, kv_heads: int, head_dim: int,
                   block_k: int, tile_q: int, num_blocks: int) -> int:
    """Bit 0: tcgen05 index stage; bit 1: tcgen05 attention for this shape;
    bit 2: the attention pairs two chunks of a selection tile per K/V stream."""
    return int(lib().fpv2_fast_path_mask(dtype_code(dtype), q_heads, kv_heads, head_dim,
                                         block_k, tile_q, num_blocks))
