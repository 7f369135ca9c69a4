"""CPU: the C-ABI library loads, exports every symbol include/*.h declares, and
rejects bad arguments with a status + message (no GPU compute is issued)."""

from __future__ import annotations

import ctypes
import re

import pytest

from conftest import REPO


def _declared_symbols() -> list[str]:
    names = []
    for h in (REPO / "include").glob("*.h"):
        names += re.findall(r"W4A16_API[^;]*?\b(w4a16_\w+)\s*\(", h.read_text(), flags=re.S)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    import build as build_mod  # package build recipe

    path = build_mod.build()
    from kernels import w4a16_moe as K

    K._lib = None
    return K.load_library()


def test_header_declares_entry_points():
    names = _declared_symbols()
    for n in ("w4a16_moe_forward", "w4a16_moe_align", "w4a16_repack", "w4a16_moe_workspace_size",
              "w4a16_last_error", "w4a16_align_buffer_len"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    for n in _declared_symbols():
        assert hasattr(lib, n), f"{n} missing from the shared library"


def test_align_buffer_len(lib):
    from oracle.moe_oracle import align_buffer_len

    for n_tok, E, bs in [(0, 256, 16), (10, 256, 16), (40960, 256, 128), (7, 3, 1), (8, 8, 16)]:
        assert lib.w4a16_align_buffer_len(n_tok, E, bs) == align_buffer_len(n_tok, E, bs)
    assert lib.w4a16_align_buffer_len(1, 1, 0) == -1


def test_workspace_size_monotone(lib):
    a = lib.w4a16_moe_workspace_size(1, 10, 256, 3072, 1024)
    b = lib.w4a16_moe_workspace_size(4096, 10, 256, 3072, 1024)
    assert 0 < a < b
    assert b % 256 == 0
    assert lib.w4a16_moe_workspace_size(1, 0, 256, 3072, 1024) == -1


def test_forward_rejects_bad_shapes(lib):
    # H not a multiple of 64 -> unsupported, before any CUDA call.
    st = lib.w4a16_moe_forward(0, 4, 100, 100, 0, 0, 0, 0, 8, 128, 0, 0, 0, 2, 0, 0, 0, 0, 0, 0)
    assert st == 2
    assert b"H % 64" in lib.w4a16_last_error()
    st = lib.w4a16_moe_forward(0, 4, 256, 256, 0, 0, 0, 0, 2000, 128, 0, 0, 0, 2, 0, 0, 0, 0, 0, 0)
    assert st == 2 and b"E=2000" in lib.w4a16_last_error()
    st = lib.w4a16_moe_forward(0, 4, 256, 256, 0, 0, 0, 0, 8, 128, 0, 0, 0, 2, 0, 0, 0, 0, 0, 0)
    assert st == 1 and b"null" in lib.w4a16_last_error()
    # M == 0 is a no-op success
    assert lib.w4a16_moe_forward(0, 0, 256, 256, 0, 0, 0, 0, 8, 128, 0, 0, 0, 2, 0, 0, 0, 0, 0, 0) == 0
    assert lib.w4a16_last_error() == b""


def test_repack_and_align_reject_bad_args(lib):
    assert lib.w4a16_repack(0, 0, 1, 16, 64, 32, 0, 0, 0) == 1
    assert lib.w4a16_repack(1, 1, 1, 15, 64, 32, 1, 1, 0) == 2
    assert lib.w4a16_repack(1, 1, 1, 16, 64, 16, 1, 1, 0) == 2
    assert lib.w4a16_moe_align(0, 0, 4, 2, 2000, 16, 0, 0, 0, 0) == 2
    assert lib.w4a16_moe_align(0, 0, 4, 0, 8, 16, 0, 0, 0, 0) == 1


def test_python_surface_fails_loudly_without_cuda():
    import torch

    from kernels import w4a16_moe as K

    ids = torch.zeros(2, 2, dtype=torch.int32)
    with pytest.raises(AssertionError):
        K.moe_align_block_size(ids, 16, 8)
    with pytest.raises(AssertionError):
        K.fused_experts_w4a16(torch.zeros(2, 64, dtype=torch.bfloat16), torch.zeros(1, 1, 1, 512, dtype=torch.uint8),
                              torch.zeros(1, 1, 1, 512, dtype=torch.uint8), torch.zeros(1), torch.zeros(1),
                              torch.zeros(2, 2), ids)


def test_library_has_no_cpu_compute_symbols(lib):
    """The library is device code + C ABI only: no host-side compute fallback."""
    out = ctypes.CDLL(str(REPO / "gb10-laguna-s-2.1-w4a16-moe_b200" / "lib" / "libw4a16moe_b200.so"))
    assert not hasattr(out, "w4a16_moe_forward_cpu")


def test_set_path_range(lib):
    for p in (0, 1, 2):
        assert lib.w4a16_set_path(p) == 0
    assert lib.w4a16_set_path(3) == 1 and b"prefill" in lib.w4a16_last_error()
    assert lib.w4a16_set_path(0) == 0


def test_align_scratch_bytes(lib):
    lib.w4a16_moe_align_scratch_bytes.restype = ctypes.c_int64
    lib.w4a16_moe_align_scratch_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64]
    assert lib.w4a16_moe_align_scratch_bytes(-1, 256) == -1
    assert lib.w4a16_moe_align_scratch_bytes(100, 2000) == -1
    assert lib.w4a16_moe_align_scratch_bytes(100, 256) == 0  # small inputs: one-CTA kernel, no scratch


def test_ep_entry_points_reject_bad_args(lib):
    vp, i64, c_int = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    lib.w4a16_ep_plan.argtypes = [vp, c_int, i64, i64, i64, i64, vp, vp, vp, vp, vp]
    lib.w4a16_ep_pack.argtypes = [vp, i64, vp, c_int, vp, i64, i64, i64, i64, vp, vp, vp, vp, vp]
    lib.w4a16_ep_combine.argtypes = [vp, vp, i64, i64, i64, vp, vp]
    # experts must divide evenly over the ranks
    assert lib.w4a16_ep_plan(1, 0, 4, 2, 10, 4, 1, 1, 1, 1, None) == 1
    assert b"divide" in lib.w4a16_last_error()
    assert lib.w4a16_ep_plan(None, 0, 4, 2, 8, 4, 1, 1, 1, 1, None) == 1  # null ids
    assert b"null" in lib.w4a16_last_error()
    # H must be a multiple of 8; M == 0 is a no-op
    assert lib.w4a16_ep_pack(1, 12, 1, 0, 1, 4, 2, 12, 2, 1, 1, 1, 1, None) == 1
    assert lib.w4a16_ep_pack(None, 256, None, 0, None, 0, 2, 256, 2, None, None, None, None, None) == 0
    assert lib.w4a16_ep_combine(1, 1, 4, 2, 12, 1, None) == 1
    assert lib.w4a16_ep_combine(None, None, 0, 2, 256, None, None) == 0
