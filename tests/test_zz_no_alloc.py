"""GPU: the allocation-free entry point matches the regular one.

w4a16_moe_forward_noalloc exists for callers that cannot allocate device
memory where they run the MoE layer (code inside another framework's memory
pool or allocator hooks, plug-in hosts that forbid allocation on the hot path,
initialisation or error paths).  It uses a static scratch array inside the
library instead of a caller workspace.  This file is named so that pytest
collects it last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    import build as build_mod

    build_mod.build()
    from kernels import w4a16_moe

    return w4a16_moe


def _noalloc(K, hidden, layer, tw, ids, out):
    lib = K.load_library()
    M, H = hidden.shape
    E = layer["w1r"].shape[0]
    I = layer["w2r"].shape[2] * 64
    st = lib.w4a16_moe_forward_noalloc(
        hidden.data_ptr(), M, H, hidden.stride(0),
        layer["w1r"].data_ptr(), layer["s1r"].data_ptr(), layer["w2r"].data_ptr(), layer["s2r"].data_ptr(),
        E, I, tw.data_ptr(), ids.data_ptr(), 1 if ids.dtype == torch.int64 else 0, ids.shape[1],
        None, 0, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return st


def test_noalloc_matches_regular_entry_point(K):
    from kernels.synthetic import make_hidden, make_layer, make_routing

    E, H, I = 64, 3072, 1024
    layer = make_layer(E, H, I, seed=3, device="cuda")
    layer["w1r"], layer["s1r"] = K.repack_weights(layer["w1_q"], layer["w1_s"])
    layer["w2r"], layer["s2r"] = K.repack_weights(layer["w2_q"], layer["w2_s"])
    lib = K.load_library()
    assert lib.w4a16_moe_noalloc_max_workspace() == 16 << 20
    # two calls in a row, of different shapes, so the second finds the first's leftovers
    for M in (16, 3, 16):
        hidden = make_hidden(M, H, seed=M, device="cuda")
        tw, ids = make_routing(M, E, 8, seed=M, device="cuda")
        ref = K.fused_experts_w4a16(hidden, layer["w1r"], layer["w2r"], layer["s1r"], layer["s2r"], tw, ids)
        out = torch.full_like(ref, float("nan"))
        st = _noalloc(K, hidden, layer, tw, ids, out)
        assert st == 0, lib.w4a16_last_error()
        torch.cuda.synchronize()
        o, r = out.float().cpu().numpy(), ref.float().cpu().numpy()
        assert np.isfinite(o).all()
        assert O.rel_frobenius(o, r) <= 1e-2
        assert O.max_abs_err(o, r) <= 1e-2 * float(np.abs(r).max())
        # no bounded device wait ran out inside the call
        i64 = ctypes.c_int64
        lib.w4a16_moe_noalloc_read_status.argtypes = [i64, i64, i64, i64, i64, ctypes.POINTER(ctypes.c_int32),
                                                      ctypes.c_void_p]
        status = ctypes.c_int32(-1)
        assert lib.w4a16_moe_noalloc_read_status(M, ids.shape[1], E, H, I, ctypes.byref(status),
                                                 torch.cuda.current_stream().cuda_stream) == 0
        assert status.value == 0


def test_noalloc_rejects_oversized_shapes(K):
    lib = K.load_library()
    M, topk, E, H, I = 4096, 10, 256, 3072, 1024
    assert lib.w4a16_moe_workspace_size(M, topk, E, H, I) > lib.w4a16_moe_noalloc_max_workspace()
    dummy = torch.empty(16, dtype=torch.uint8, device="cuda")
    p = dummy.data_ptr()
    st = lib.w4a16_moe_forward_noalloc(p, M, H, H, p, p, p, p, E, I, p, p, 0, topk, None, 0, p, None)
    assert st == 2
    assert b"16 MiB" in lib.w4a16_last_error()
