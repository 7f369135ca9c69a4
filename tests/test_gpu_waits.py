"""Bounded device waits: a wait that runs out reports an error status and
leaves the GPU usable.  The multi-CTA align kernel's grid barrier is made to
time out on purpose through the library's test hook (one CTA withholds its
arrival, the others wait ~10 us), with no fault, trap or unbounded wait; the
timeout must appear in w4a16_moe_align_read_status, and the same scratch must
give bit-exact results on the next normal call.  The fused decode kernel's
per-expert readiness wait is made to run out the same way (CTA 0 publishes
none of its w13 items, the w2 items wait ~10 us): the call returns, the error
bit is reported, and the next normal call is bit-exact."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

ALIGN_TIMEOUT_BIT = 1 << 16


@pytest.fixture(scope="module")
def lib():
    import build as build_mod

    build_mod.build()
    from kernels import w4a16_moe

    lib = w4a16_moe.load_library()
    lib.w4a16_set_wait_test.restype = ctypes.c_int
    lib.w4a16_set_wait_test.argtypes = [ctypes.c_int]
    lib.w4a16_moe_align_read_status.restype = ctypes.c_int
    lib.w4a16_moe_align_read_status.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32), ctypes.c_void_p]
    yield lib
    lib.w4a16_set_wait_test(0)


def _align(lib, ids, bs, E, scratch):
    M, topk = ids.shape
    P = int(lib.w4a16_align_buffer_len(M * topk, E, bs))
    s = torch.full((P,), -7, dtype=torch.int32, device="cuda")
    e = torch.full((P // bs,), -7, dtype=torch.int32, device="cuda")
    n = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    rc = lib.w4a16_moe_align_ex(ids.data_ptr(), 0, M, topk, E, bs, s.data_ptr(), e.data_ptr(), n.data_ptr(),
                                scratch.data_ptr(), scratch.numel(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.w4a16_last_error()
    return s, e, n


def _status(lib, scratch):
    out = ctypes.c_int32(-1)
    assert lib.w4a16_moe_align_read_status(scratch.data_ptr(), ctypes.byref(out),
                                           torch.cuda.current_stream().cuda_stream) == 0
    return out.value


def test_align_barrier_timeout_is_reported(lib):
    M, topk, E, bs = 4096, 10, 256, 16
    g = torch.Generator().manual_seed(11)
    ids_cpu = torch.topk(torch.randn(M, E, generator=g), k=topk, dim=-1).indices.to(torch.int32)
    ids = ids_cpu.cuda()
    sb = int(lib.w4a16_moe_align_scratch_bytes(M * topk, E))
    assert sb > 0, "this size must use the multi-CTA kernel"
    scratch = torch.zeros(sb, dtype=torch.uint8, device="cuda")

    assert lib.w4a16_set_wait_test(1) == 0
    try:
        s, _, _ = _align(lib, ids, bs, E, scratch)
        torch.cuda.synchronize()
    finally:
        assert lib.w4a16_set_wait_test(0) == 0
    assert _status(lib, scratch) & ALIGN_TIMEOUT_BIT
    # the timed-out call wrote no sorted ids past the untouched fill
    assert int((s == -7).sum()) > 0

    # the context is still usable and the scratch works again after the query
    s, e, n = _align(lib, ids, bs, E, scratch)
    torch.cuda.synchronize()
    assert _status(lib, scratch) == 0
    rs, re_, rn = O.align_block_size(ids_cpu.numpy(), bs, E)
    np.testing.assert_array_equal(s.cpu().numpy(), rs)
    np.testing.assert_array_equal(e.cpu().numpy(), re_)
    np.testing.assert_array_equal(n.cpu().numpy(), rn)


DECODE_READY_WAIT_BIT = 4


def test_decode_readiness_timeout_is_reported(lib):
    from kernels import w4a16_moe as K
    from kernels.synthetic import make_hidden, make_layer, make_routing

    E, H, I, M = 256, 3072, 1024, 1
    layer = make_layer(E, H, I, seed=0, device="cuda")
    w1r, s1r = K.repack_weights(layer["w1_q"], layer["w1_s"])
    w2r, s2r = K.repack_weights(layer["w2_q"], layer["w2_s"])
    del layer
    hidden = make_hidden(M, H, device="cuda")
    tw, ids = make_routing(M, E, 10, device="cuda")
    ref = K.fused_experts_w4a16(hidden, w1r, w2r, s1r, s2r, tw, ids).clone()
    torch.cuda.synchronize()
    assert K.read_status((M, H), 10, E, I) == 0

    assert lib.w4a16_set_wait_test(2) == 0
    try:
        K.fused_experts_w4a16(hidden, w1r, w2r, s1r, s2r, tw, ids)
        torch.cuda.synchronize()
    finally:
        assert lib.w4a16_set_wait_test(0) == 0
    assert K.read_status((M, H), 10, E, I) & DECODE_READY_WAIT_BIT

    # counters were reset by the timed-out call: the next one is exact again
    again = K.fused_experts_w4a16(hidden, w1r, w2r, s1r, s2r, tw, ids)
    torch.cuda.synchronize()
    assert K.read_status((M, H), 10, E, I) == 0
    assert torch.equal(again, ref)
