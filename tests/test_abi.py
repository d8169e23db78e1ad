"""C-ABI checks that need no GPU: the library loads, exports every function that
include/duplex_b200.h declares, and rejects bad arguments before touching CUDA."""

import ctypes
import re
from pathlib import Path

import pytest

from duplex import _build, _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "duplex_b200.h"


@pytest.fixture(scope="module")
def lib():
    _build.build()
    return _lib.load()


def declared():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(duplex_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_bound_api():
    assert set(declared()) == set(_lib.exported_symbols())


def test_every_declared_symbol_is_exported(lib):
    for name in declared():
        assert hasattr(lib, name), name


def test_version_and_errors(lib):
    assert lib.duplex_version() >= 100
    for code in range(0, 7):
        assert lib.duplex_error_string(code)
    assert b"unknown" in lib.duplex_error_string(99)


def test_bad_arguments_are_rejected_without_cuda(lib):
    null = None
    # null pointers
    assert lib.duplex_dq_gemv(null, 0, 0, null, null, null, 0, 1, 16, 16, 64, 32, null, 1, null,
                              null, null) == 1
    assert lib.duplex_unpack4(null, 1, 1, 8, null, null) == 1
    assert lib.duplex_dequant(null, null, 0, null, 1, 64, 32, null, 0, null) == 1
    n = ctypes.c_size_t()
    assert lib.duplex_moe_workspace_bytes(0, 128, 2048, 768, 8, ctypes.byref(n)) == 1
    assert lib.duplex_moe_workspace_bytes(1, 128, 2048, 768, 8, ctypes.byref(n)) == 0
    assert n.value > 0


def test_unsupported_shapes_are_rejected(lib):
    # fake but aligned addresses: validation must reject before any launch
    p = ctypes.c_void_p(1 << 20)
    # K not a multiple of 32
    assert lib.duplex_packed_linear(p, 0, 1, 48, p, p, None, 0, 16, 16, 48, 32, None, None, 0, p,
                                    16, 0.0, 0, None) == 6
    # rows per expert not a multiple of 16
    assert lib.duplex_packed_linear(p, 0, 1, 64, p, p, None, 0, 10, 10, 64, 32, None, None, 0, p,
                                    10, 0.0, 0, None) == 6
    # batch > 8
    assert lib.duplex_packed_linear(p, 0, 9, 64, p, p, None, 0, 16, 16, 64, 32, None, None, 0, p,
                                    16, 0.0, 0, None) == 1
    # misaligned activation pointer
    q = ctypes.c_void_p((1 << 20) + 8)
    assert lib.duplex_packed_linear(q, 0, 1, 64, p, p, None, 0, 16, 16, 64, 32, None, None, 0, p,
                                    16, 0.0, 0, None) == 2
    # bad dtype
    assert lib.duplex_packed_linear(p, 0, 1, 64, p, p, None, 7, 16, 16, 64, 32, None, None, 0, p,
                                    16, 0.0, 0, None) == 3
    # router: T > 8, top_k > E
    assert lib.duplex_moe_route(p, 0, 9, p, None, 128, 2048, 8, 1, None, None, p, 1 << 30, 0.0, 0,
                                None) == 1
    assert lib.duplex_moe_route(p, 0, 1, p, None, 4, 2048, 8, 1, None, None, p, 1 << 30, 0.0, 0,
                                None) == 1
    # workspace too small
    assert lib.duplex_moe_route(p, 0, 1, p, None, 128, 2048, 8, 1, None, None, p, 16, 0.0, 0,
                                None) == 4


def test_python_wrappers_refuse_cpu_tensors():
    import torch
    from duplex.streaming.fused_packed_moe import unpack4
    from duplex.streaming.triton_dequant_gemv import dequant_gemv
    with pytest.raises(_lib.DuplexError):
        unpack4(torch.zeros(2, 4, dtype=torch.int32), 32)
    with pytest.raises(_lib.DuplexError):
        dequant_gemv(torch.zeros(64, dtype=torch.float16), torch.zeros(1, 16, 8, dtype=torch.int32),
                     torch.ones(1, 16, 2, dtype=torch.float16), torch.zeros(1, dtype=torch.int32))
