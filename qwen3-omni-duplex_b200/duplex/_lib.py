"""ctypes binding of the C ABI in include/duplex_b200.h (libduplex_b200.so).

This is the same binding a maintainer of the reference would add: plain device
pointers (tensor.data_ptr()), sizes, dtype codes and the current CUDA stream.
There is no fallback: if the library is missing or fails to load, every
product entry point raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("DUPLEX_B200_LIB", _PKG / "libduplex_b200.so"))

DTYPE_F16, DTYPE_BF16, DTYPE_F32 = 0, 1, 2
DEVERR_EXPERT, DEVERR_TIMEOUT = 1, 2

_c_int, _c_i32, _c_i64, _c_ptr, _c_size, _c_f32 = (ctypes.c_int, ctypes.c_int32, ctypes.c_int64,
                                                   ctypes.c_void_p, ctypes.c_size_t,
                                                   ctypes.c_float)

_SIGNATURES = {
    "duplex_version": ([], _c_int),
    "duplex_error_string": ([_c_int], ctypes.c_char_p),
    "duplex_last_cuda_error": ([], _c_int),
    "duplex_unpack4": ([_c_ptr, _c_i64, _c_i32, _c_i32, _c_ptr, _c_ptr], _c_int),
    "duplex_dequant": ([_c_ptr, _c_ptr, _c_int, _c_ptr, _c_i64, _c_i32, _c_i32, _c_ptr, _c_int,
                        _c_ptr], _c_int),
    "duplex_tile_record_bytes": ([_c_i32, _c_i32, _c_int, ctypes.POINTER(ctypes.c_size_t)], _c_int),
    "duplex_repack_tiles": ([_c_ptr, _c_ptr, _c_ptr, _c_int, _c_i32, _c_i32, _c_i32, _c_i32,
                             _c_i32, _c_ptr, _c_size, _c_ptr], _c_int),
    "duplex_dq_gemv": ([_c_ptr, _c_int, _c_i64, _c_ptr, _c_int, _c_int, _c_i32, _c_i32, _c_i32,
                        _c_i32, _c_ptr, _c_i32, _c_ptr, _c_ptr, _c_ptr], _c_int),
    "duplex_packed_linear": ([_c_ptr, _c_int, _c_i32, _c_i64, _c_ptr, _c_int, _c_int, _c_i32,
                              _c_i32, _c_i32, _c_ptr, _c_ptr, _c_i64, _c_ptr, _c_i64, _c_f32,
                              _c_int, _c_ptr], _c_int),
    "duplex_moe_workspace_bytes": ([_c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
                                    ctypes.POINTER(ctypes.c_size_t)], _c_int),
    "duplex_moe_route": ([_c_ptr, _c_int, _c_i32, _c_ptr, _c_ptr, _c_i32, _c_i32, _c_i32, _c_i32,
                          _c_ptr, _c_ptr, _c_ptr, _c_size, _c_f32, _c_int, _c_ptr], _c_int),
    "duplex_moe_forward": ([_c_ptr, _c_int, _c_i32, _c_ptr, _c_ptr, _c_i32, _c_i32, _c_i32,
                            _c_i32, _c_i32, _c_ptr, _c_ptr, _c_int, _c_int, _c_i32, _c_ptr,
                            _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_size, _c_ptr, _c_f32, _c_int,
                            _c_ptr], _c_int),
    "duplex_host_alloc": ([_c_size, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p)],
                          _c_int),
    "duplex_host_free": ([_c_ptr], _c_int),
    "duplex_moe_stage_bytes": ([_c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_int,
                                ctypes.POINTER(ctypes.c_size_t)], _c_int),
    "duplex_moe_forward_staged": ([_c_ptr, _c_int, _c_i32, _c_ptr, _c_ptr, _c_i32, _c_i32, _c_i32,
                                   _c_i32, _c_i32, _c_ptr, _c_ptr, _c_int, _c_int, _c_i32, _c_ptr,
                                   _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_size, _c_ptr, _c_size, _c_ptr,
                                   _c_f32, _c_int, _c_ptr], _c_int),
    "duplex_moe_noalloc_scratch_bytes": ([], _c_size),
    "duplex_moe_forward_noalloc": ([_c_ptr, _c_int, _c_i32, _c_ptr, _c_ptr, _c_i32, _c_i32,
                                    _c_i32, _c_i32, _c_i32, _c_ptr, _c_ptr, _c_int, _c_int,
                                    _c_i32, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_f32,
                                    _c_int, _c_ptr], _c_int),
    "duplex_moe_grouped_workspace_bytes": ([_c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
                                            _c_int, ctypes.POINTER(ctypes.c_size_t)], _c_int),
    "duplex_moe_grouped": ([_c_ptr, _c_int, _c_i32, _c_ptr, _c_ptr, _c_ptr, _c_i32, _c_i32,
                            _c_i32, _c_i32, _c_i32, _c_ptr, _c_ptr, _c_int, _c_int, _c_i32,
                            _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_size, _c_ptr, _c_ptr],
                           _c_int),
    "duplex_moe_route_grouped": ([_c_ptr, _c_int, _c_i32, _c_ptr, _c_ptr, _c_ptr, _c_i32, _c_i32,
                                  _c_i32, _c_i32, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_ptr, _c_size,
                                  _c_ptr, _c_ptr], _c_int),
    "duplex_moe_experts_grouped_workspace_bytes": ([_c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
                                                    _c_i32, _c_int, ctypes.POINTER(ctypes.c_size_t)],
                                                   _c_int),
    "duplex_moe_experts_grouped": ([_c_ptr, _c_int, _c_i32, _c_i64, _c_ptr, _c_ptr, _c_i32, _c_i32,
                                    _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_ptr, _c_ptr, _c_int,
                                    _c_int, _c_i32, _c_ptr, _c_ptr, _c_int, _c_ptr, _c_size, _c_ptr,
                                    _c_ptr], _c_int),
    "duplex_tc_records_bytes": ([_c_i32, _c_i32, _c_i32, _c_i32, _c_int, _c_i32,
                                 ctypes.POINTER(ctypes.c_size_t)], _c_int),
    "duplex_repack_tc_records": ([_c_ptr, _c_ptr, _c_ptr, _c_int, _c_i32, _c_i32, _c_i32, _c_i32,
                                  _c_i32, _c_ptr, _c_size, _c_ptr], _c_int),
    "duplex_moe_grouped_tc_workspace_bytes": ([_c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
                                               _c_int, ctypes.POINTER(ctypes.c_size_t)], _c_int),
    "duplex_moe_grouped_tc": ([_c_ptr, _c_int, _c_i32, _c_ptr, _c_ptr, _c_ptr, _c_i32, _c_i32,
                               _c_i32, _c_i32, _c_i32, _c_ptr, _c_ptr, _c_int, _c_int, _c_i32,
                               _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_size, _c_ptr, _c_ptr],
                              _c_int),
    "duplex_moe_experts_grouped_tc_workspace_bytes": ([_c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
                                                       _c_i32, _c_i32, _c_int,
                                                       ctypes.POINTER(ctypes.c_size_t)], _c_int),
    "duplex_moe_experts_grouped_tc": ([_c_ptr, _c_int, _c_i32, _c_i64, _c_ptr, _c_ptr, _c_i32,
                                       _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_ptr,
                                       _c_ptr, _c_int, _c_int, _c_i32, _c_ptr, _c_ptr, _c_int,
                                       _c_ptr, _c_size, _c_ptr, _c_ptr], _c_int),
    "duplex_stack_workspace_bytes": ([_c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
                                      ctypes.POINTER(ctypes.c_size_t)], _c_int),
    "duplex_stack_forward": ([_c_ptr, _c_i32, _c_i32, _c_i32, _c_ptr, _c_ptr, _c_int, _c_int,
                              _c_int, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
                              _c_i32, _c_i32, _c_f32, _c_ptr, _c_size, _c_i64, _c_i32, _c_ptr,
                              _c_ptr], _c_int),
    "duplex_ep_dispatch_pack": ([_c_ptr, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, _c_i64, _c_ptr,
                                 _c_ptr, _c_ptr], _c_int),
    "duplex_ep_combine": ([_c_ptr, _c_ptr, _c_i32, _c_i32, _c_i32, _c_ptr, _c_ptr, _c_int, _c_ptr],
                          _c_int),
    "duplex_ipc_handle_bytes": ([], _c_int),
    "duplex_ipc_alloc": ([_c_size, ctypes.POINTER(ctypes.c_void_p), _c_ptr], _c_int),
    "duplex_ipc_open": ([_c_ptr, ctypes.POINTER(ctypes.c_void_p)], _c_int),
    "duplex_ipc_close": ([_c_ptr], _c_int),
    "duplex_ipc_free": ([_c_ptr], _c_int),
    "duplex_ep_dispatch_peer": ([_c_ptr, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i64,
                                 _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr], _c_int),
    "duplex_ep_put_peer": ([_c_ptr, _c_i64, _c_i32, _c_i32, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr],
                           _c_int),
    "duplex_ep_wait": ([_c_ptr, _c_ptr, _c_i32, _c_i64, _c_ptr, _c_ptr], _c_int),
    "duplex_talker_moe_workspace_bytes": ([_c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
                                           ctypes.POINTER(ctypes.c_size_t)], _c_int),
    "duplex_talker_moe_forward": ([_c_ptr, _c_int, _c_i32, _c_ptr, _c_i32, _c_i32, _c_i32, _c_i32,
                                   _c_i32, _c_ptr, _c_ptr, _c_int, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
                                   _c_ptr, _c_i32, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_size,
                                   _c_ptr, _c_ptr], _c_int),
    "duplex_gate_records_bytes": ([_c_i32, _c_i32, ctypes.POINTER(ctypes.c_size_t)], _c_int),
    "duplex_repack_gate_records": ([_c_ptr, _c_int, _c_i32, _c_i32, _c_ptr, _c_size, _c_ptr],
                                   _c_int),
    "duplex_down_slices_bytes": ([_c_i32, _c_i32, _c_i32, _c_i32, _c_int,
                                  ctypes.POINTER(ctypes.c_size_t)], _c_int),
    "duplex_repack_down_slices": ([_c_ptr, _c_ptr, _c_ptr, _c_int, _c_i32, _c_i32, _c_i32, _c_i32,
                                   _c_ptr, _c_size, _c_ptr], _c_int),
}


class StackLayer(ctypes.Structure):
    """duplex_stack_layer of include/duplex_b200.h (device pointers of one layer)."""
    _fields_ = [("qkv_tiles", ctypes.c_void_p), ("o_tiles", ctypes.c_void_p),
                ("gate_w", ctypes.c_void_p), ("gate_b", ctypes.c_void_p),
                ("gu_tiles", ctypes.c_void_p), ("dn_tiles", ctypes.c_void_p)]


_lib = None


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load (once) and type the shared library; raise loudly if it is unavailable."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"duplex_b200: {p} not found. Build it with `python -m duplex._build` "
            "(or __graft_entry__.build()); there is no non-CUDA fallback.")
    lib = ctypes.CDLL(str(p))
    for name, (args, res) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    if path is None:
        _lib = lib
    return lib


_torch_ops_loaded = False


def load_torch_ops():
    """Register the TORCH_LIBRARY(duplex_b200) ops (libduplex_torch_ops.so, in-tree):
    afterwards torch.ops.duplex_b200.<op> call the same C entry points."""
    global _torch_ops_loaded
    if not _torch_ops_loaded:
        load()
        p = _PKG / "libduplex_torch_ops.so"
        if not p.exists():
            raise RuntimeError(f"duplex_b200: {p} not found; build it with duplex._build")
        torch.ops.load_library(str(p))
        _torch_ops_loaded = True
    return torch.ops.duplex_b200


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


class DuplexError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc != 0:
        lib = load()
        msg = lib.duplex_error_string(rc).decode()
        extra = f" (cudaError {lib.duplex_last_cuda_error()})" if rc == 5 else ""
        raise DuplexError(f"{what} failed: status {rc}: {msg}{extra}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float16:
        return DTYPE_F16
    if dt == torch.bfloat16:
        return DTYPE_BF16
    if dt == torch.float32:
        return DTYPE_F32
    raise DuplexError(f"unsupported dtype {dt}")


def require_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise DuplexError("duplex_b200 kernels take CUDA tensors only (no CPU path)")


def aligned(t: torch.Tensor) -> torch.Tensor:
    """Contiguous and 16-byte aligned (copies only when needed)."""
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t
