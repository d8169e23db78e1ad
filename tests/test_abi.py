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
    for code in range(0, 8):
        assert lib.duplex_error_string(code)
    assert b"unknown" in lib.duplex_error_string(99)


def test_bad_arguments_are_rejected_without_cuda(lib):
    null = None
    # null pointers
    assert lib.duplex_dq_gemv(null, 0, 0, null, 0, 0, 1, 16, 64, 32, null, 1, null, null,
                              null) == 1
    assert lib.duplex_repack_tiles(null, null, null, 0, 1, 16, 64, 32, 0, null, 0, null) == 1
    assert lib.duplex_tile_record_bytes(2048, 128, 1, ctypes.byref(n := ctypes.c_size_t())) == 0
    assert n.value == 16384 + 16 * 32 + 16 * 8
    assert lib.duplex_tile_record_bytes(768, 128, 0, ctypes.byref(n)) == 0
    assert n.value == 6144 + 6 * 32 + 64   # padded to 128 bytes
    assert lib.duplex_tile_record_bytes(2048, 96, 0, ctypes.byref(n)) == 6
    assert lib.duplex_unpack4(null, 1, 1, 8, null, null) == 1
    assert lib.duplex_dequant(null, null, 0, null, 1, 64, 32, null, 0, null) == 1
    n = ctypes.c_size_t()
    assert lib.duplex_moe_workspace_bytes(0, 128, 2048, 768, 8, ctypes.byref(n)) == 1
    assert lib.duplex_moe_workspace_bytes(1, 128, 2048, 768, 8, ctypes.byref(n)) == 0
    assert n.value > 0


def test_unsupported_shapes_are_rejected(lib):
    # fake but aligned addresses: validation must reject before any launch
    p = ctypes.c_void_p(1 << 20)

    def lin(x=p, act=0, B=1, xs=64, sdt=0, R=16, K=64, group=32):
        return lib.duplex_packed_linear(x, act, B, xs, p, sdt, 0, R, K, group, None, None, 0, p,
                                        R, 0.0, 0, None)

    assert lin(K=48, xs=48) == 6                   # K not a multiple of 32
    assert lin(group=48) == 6                      # group neither 32 nor 64 * 2^k
    assert lin(B=9) == 1                           # batch > 8
    assert lin(x=ctypes.c_void_p((1 << 20) + 8)) == 2   # misaligned activations
    assert lin(sdt=7) == 3                         # bad scale dtype
    # router: T > 8, top_k > E
    assert lib.duplex_moe_route(p, 0, 9, p, None, 128, 2048, 8, 1, None, None, p, 1 << 30, 0.0, 0,
                                None) == 1
    assert lib.duplex_moe_route(p, 0, 1, p, None, 4, 2048, 8, 1, None, None, p, 1 << 30, 0.0, 0,
                                None) == 1
    # workspace too small
    assert lib.duplex_moe_route(p, 0, 1, p, None, 128, 2048, 8, 1, None, None, p, 16, 0.0, 0,
                                None) == 4


def test_grouped_moe_rejects_before_any_launch(lib):
    n = ctypes.c_size_t()

    def wsb(T=256, E=128, H=2048, I=768, k=8, group=128, zp=1):
        return lib.duplex_moe_grouped_workspace_bytes(T, E, H, I, k, group, zp, ctypes.byref(n))

    assert wsb() == 0 and n.value > 256 * 8 * 2048 * 4   # one fp32 row per (token, slot)
    assert wsb(T=512) == 0
    assert wsb(T=513) == 1                         # more tokens than one call takes
    assert wsb(E=257) == 1 and wsb(k=9) == 1
    assert wsb(group=32) == 6                      # groups below 64 columns
    assert wsb(group=96) == 6
    assert wsb(H=4096) == 6                        # one unit's token rows + 2 slots > 227 KB
    assert wsb(I=1536) == 6
    assert wsb(I=1024) == 0
    p = ctypes.c_void_p(1 << 20)
    big = 1 << 30

    def grouped(x=p, T=64, group=128, ws=big, logits=None, gate=p, act=0, sdt=0):
        return lib.duplex_moe_grouped(x, act, T, gate, None, logits, 128, 2048, 768, 8, 1, p, p,
                                      sdt, 1, group, None, p, None, None, p, ws, p, None)

    assert grouped(T=0) == 1 and grouped(T=513) == 1
    assert grouped(gate=None) == 1                 # neither a gate nor logits
    assert grouped(x=ctypes.c_void_p((1 << 20) + 4)) == 2
    assert grouped(logits=ctypes.c_void_p((1 << 20) + 4)) == 2
    assert grouped(sdt=1) == 3 and grouped(act=2, sdt=2) == 3
    assert grouped(group=32) == 6
    assert grouped(ws=16) == 4


def test_tc_path_sizes_and_rejections(lib):
    """Tensor-core records and the tcgen05 entry points: sizes, and every geometry they do
    not take rejected before any launch."""
    n = ctypes.c_size_t()

    def rb(E=128, R=1536, K=2048, group=128, zp=1, pair=1):
        return lib.duplex_tc_records_bytes(E, R, K, group, zp, pair, ctypes.byref(n))

    assert rb() == 0 and n.value == 128 * 12 * 16 * (8192 + 256 + 128)   # Thinker gate|up
    assert rb(R=2048, K=768, pair=0) == 0 and n.value == 128 * 16 * 6 * (8192 + 256 + 128)
    assert rb(zp=0) == 0 and n.value == 128 * 12 * 16 * (8192 + 256)
    assert rb(group=64) == 6 and rb(K=2000) == 6 and rb(R=1000) == 6
    assert rb(E=0) == 1

    def wsb(T=256, E=128, H=2048, I=768, k=8, group=128):
        return lib.duplex_moe_grouped_tc_workspace_bytes(T, E, H, I, k, group, 1, ctypes.byref(n))

    assert wsb() == 0 and n.value > 256 * 8 * 2048 * 4
    assert wsb(T=513) == 1 and wsb(k=9) == 1
    assert wsb(group=64) == 6                      # one scale group per 128-column chunk
    assert wsb(H=2176) == 6 and wsb(I=640) == 6    # whole two-chunk stages only
    assert wsb(I=512) == 0
    assert lib.duplex_moe_experts_grouped_tc_workspace_bytes(256, 16, 128, 2048, 768, 8, 128, 1,
                                                             ctypes.byref(n)) == 0
    assert lib.duplex_moe_experts_grouped_tc_workspace_bytes(256, 16, 8, 2048, 768, 8, 128, 1,
                                                             ctypes.byref(n)) == 1  # E_total < E_local
    p = ctypes.c_void_p(1 << 20)

    def tc(x=p, T=64, group=128, ws=1 << 30, act=0, sdt=0):
        return lib.duplex_moe_grouped_tc(x, act, T, p, None, None, 128, 2048, 768, 8, 1, p, p, sdt, 1,
                                         group, None, p, None, None, p, ws, p, None)

    assert tc(T=0) == 1 and tc(sdt=1) == 3 and tc(group=64) == 6 and tc(ws=16) == 4
    assert tc(x=ctypes.c_void_p((1 << 20) + 4)) == 2
    pk = ctypes.c_void_p(1 << 20)
    assert lib.duplex_repack_tc_records(pk, pk, None, 0, 1, 128, 256, 128, 0, pk, 16, None) == 4  # too small


def test_python_wrappers_refuse_cpu_tensors():
    import torch
    from duplex.streaming.fused_packed_moe import unpack4
    from duplex.streaming.triton_dequant_gemv import dequant_gemv
    with pytest.raises(_lib.DuplexError):
        unpack4(torch.zeros(2, 4, dtype=torch.int32), 32)
    with pytest.raises(_lib.DuplexError):
        dequant_gemv(torch.zeros(64, dtype=torch.float16), torch.zeros(1, 16, 8, dtype=torch.int32),
                     torch.ones(1, 16, 2, dtype=torch.float16), torch.zeros(1, dtype=torch.int32))


def test_torch_library_ops_are_registered():
    """TORCH_LIBRARY(duplex_b200) registers every op (schemas only; no GPU call)."""
    from duplex import _build
    _build.build_torch_ops()
    ops = _lib.load_torch_ops()
    import torch
    for name in ("unpack4", "dequant", "dequant_gemv", "packed_linear", "moe_forward",
                 "moe_grouped", "ep_dispatch", "ep_combine", "moe_route", "talker_moe"):
        op = getattr(ops, name)
        assert isinstance(op.default, torch._ops.OpOverload), name
    assert "Tensor(a!) send" in str(ops.ep_dispatch.default._schema)


def test_host_resident_staging_sizes_and_rejections(lib):
    """duplex_moe_stage_bytes: the staged plan plus min(T * top_k, E) experts' gate|up and
    down records; duplex_moe_forward_staged rejects bad arguments before any launch."""
    def rec(K, zp):
        n = ctypes.c_size_t()
        assert lib.duplex_tile_record_bytes(K, 128, zp, ctypes.byref(n)) == 0
        return n.value

    def up256(v):
        return -(-v // 256) * 256

    H, I, E, k = 2048, 768, 128, 8
    gu, dn = (2 * I // 16) * rec(H, 1), (H // 16) * rec(I, 1)
    plan = up256(16 + 64 * 4 + 64 * 4 + 64 * 8 * 4)      # MoePlan
    n = ctypes.c_size_t()
    for T, slots in ((1, 8), (8, 64)):
        assert lib.duplex_moe_stage_bytes(T, E, H, I, k, 128, 1, ctypes.byref(n)) == 0
        assert n.value == plan + up256(slots * gu) + up256(slots * dn)
    # fewer experts than T * top_k: one slot per expert
    assert lib.duplex_moe_stage_bytes(8, 16, 256, 128, 4, 32, 0, ctypes.byref(n)) == 0
    r256, r128 = ctypes.c_size_t(), ctypes.c_size_t()
    assert lib.duplex_tile_record_bytes(256, 32, 0, ctypes.byref(r256)) == 0
    assert lib.duplex_tile_record_bytes(128, 32, 0, ctypes.byref(r128)) == 0
    assert n.value == plan + up256(16 * 16 * r256.value) + up256(16 * 16 * r128.value)
    assert lib.duplex_moe_stage_bytes(9, E, H, I, k, 128, 1, ctypes.byref(n)) == 1
    assert lib.duplex_moe_stage_bytes(1, E, H, I, k, 96, 1, ctypes.byref(n)) == 6

    p = ctypes.c_void_p(1 << 20)          # aligned, never dereferenced: every call rejects
    odd = ctypes.c_void_p((1 << 20) + 8)
    big = 1 << 40

    def staged(T=1, out=p, stage=p, stage_bytes=big, ws=p, ws_bytes=big, gu=p):
        return lib.duplex_moe_forward_staged(p, 0, T, p, None, E, H, I, k, 1, gu, p, 0, 1, 128,
                                             None, out, None, None, ws, ws_bytes, stage,
                                             stage_bytes, None, 0.0, 0, None)

    assert staged(stage=None) == 1                      # DUPLEX_ERR_ARG
    assert staged(T=9) == 1
    assert staged(out=odd) == 2                         # DUPLEX_ERR_ALIGN
    assert staged(gu=odd) == 2
    assert staged(stage_bytes=1024) == 4                # DUPLEX_ERR_WORKSPACE
    assert staged(ws_bytes=16) == 4                     # the router's workspace check
    assert lib.duplex_host_alloc(0, ctypes.byref(ctypes.c_void_p()),
                                 ctypes.byref(ctypes.c_void_p())) == 1
    assert lib.duplex_host_free(None) == 1


def test_expert_parallel_entry_points_reject_before_any_launch(lib):
    """The exchange entry points (dispatch pack, peer dispatch / put / wait, combine, CUDA
    IPC) reject bad arguments with a status and touch no device."""
    p = ctypes.c_void_p(1 << 20)          # aligned, never dereferenced: every call rejects
    null = None
    assert lib.duplex_ipc_handle_bytes() == 64
    assert lib.duplex_ipc_alloc(0, ctypes.byref(ctypes.c_void_p()), p) == 1
    assert lib.duplex_ipc_open(null, ctypes.byref(ctypes.c_void_p())) == 1
    # dispatch pack: T over 512, experts not split evenly, rows not a multiple of 16 B
    assert lib.duplex_ep_dispatch_pack(p, 4112, 513, 8, 128, 2, 4096, p, p, null) == 1
    assert lib.duplex_ep_dispatch_pack(p, 4112, 32, 8, 128, 3, 4096, p, p, null) == 1
    assert lib.duplex_ep_dispatch_pack(p, 4104, 32, 8, 128, 2, 4096, p, p, null) == 2
    # peer dispatch: rank outside the group, missing flags
    assert lib.duplex_ep_dispatch_peer(p, 4112, 32, 8, 128, 2, 2, 4096, p, p, p, p, p, null) == 1
    assert lib.duplex_ep_dispatch_peer(p, 4112, 32, 8, 128, 2, 0, 4096, p, p, null, p, p,
                                       null) == 1
    # put: blocks under 16 B or not a multiple of 16 B
    assert lib.duplex_ep_put_peer(p, 8, 2, 0, p, p, p, p, null) == 1
    assert lib.duplex_ep_put_peer(p, 24, 2, 0, p, p, p, p, null) == 2
    # wait: no error word, no ranks
    assert lib.duplex_ep_wait(p, p, 2, 0, null, null) == 1
    assert lib.duplex_ep_wait(p, p, 0, 0, p, null) == 1
    # combine: H not a multiple of 4, unsupported activation dtype
    assert lib.duplex_ep_combine(p, p, 32, 2, 2046, null, p, 0, null) == 1
    assert lib.duplex_ep_combine(p, p, 32, 2, 2048, null, p, 7, null) == 3


def test_plain_c_host_links_and_calls_the_library(lib, tmp_path):
    """include/duplex_b200.h compiles as C99 and a C program links the library and gets
    its answers (tests/c/abi_smoke.c): the boundary needs no C++ or Python on the host."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    src = Path(__file__).resolve().parent / "c" / "abi_smoke.c"
    so = Path(_lib.__file__).resolve().parent / "libduplex_b200.so"
    exe = tmp_path / "abi_smoke"
    r = subprocess.run([cc, "-std=c99", "-Wall", "-Werror", f"-I{HEADER.parent}", str(src),
                        "-o", str(exe), f"-L{so.parent}", "-lduplex_b200",
                        f"-Wl,-rpath,{so.parent}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
