"""Expert-parallel exchange kernels on the GPU (through the C ABI):
plan / pack / combine bit-exact against the oracle, an expert-parallel layer
emulated on one GPU against the single-GPU forward, and -- with two or more
GPUs -- the NCCL path end to end."""

from __future__ import annotations

import socket
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import ep_oracle as EO
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ep():
    from kernels import ep as mod

    return mod


def _routing(M, E, k, seed, int64=False):
    g = torch.Generator().manual_seed(seed)
    ids = torch.topk(torch.randn(M, E, generator=g), k=k, dim=-1).indices
    tw = torch.softmax(torch.randn(M, k, generator=g), dim=-1)
    return tw, ids.to(torch.int64 if int64 else torch.int32)


@pytest.mark.parametrize("M,E,k,world,int64", [(1, 256, 10, 8, False), (300, 256, 10, 4, True),
                                               (5000, 256, 10, 8, False), (64, 8, 2, 2, False),
                                               (7, 16, 3, 1, False), (0, 16, 2, 2, False)])
def test_plan_pack_bitexact(ep, M, E, k, world, int64):
    from kernels import w4a16_moe as K

    tw, ids = _routing(M, E, k, seed=M + world, int64=int64)
    H = 256
    x = torch.randn(M, H, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    dev = torch.device("cuda")
    lib = ep._lib()
    idsd, twd, xd = ids.to(dev), tw.to(dev), x.to(dev)
    counts = torch.empty(world, dtype=torch.int32, device=dev)
    offsets = torch.empty(world + 1, dtype=torch.int32, device=dev)
    send_tok = torch.full((max(M * world, 1),), -7, dtype=torch.int32, device=dev)
    tok_row = torch.empty(max(M * world, 1), dtype=torch.int32, device=dev)
    K._check(lib.w4a16_ep_plan(idsd.data_ptr(), int(int64), M, k, E, world, counts.data_ptr(), offsets.data_ptr(),
                               send_tok.data_ptr(), tok_row.data_ptr(), None), "plan")
    rc, ro, rs, rt = EO.plan(ids.numpy(), E, world)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(counts.cpu().numpy(), rc)
    np.testing.assert_array_equal(offsets.cpu().numpy(), ro)
    n = int(ro[-1])
    np.testing.assert_array_equal(send_tok.cpu().numpy()[:n], rs)
    if M:
        np.testing.assert_array_equal(tok_row.cpu().numpy()[: M * world].reshape(M, world), rt)
    pl = ep.Plan(rc.tolist(), rc.tolist(), offsets, send_tok, tok_row)
    if M:
        x_send, meta = ep.pack(xd, twd, idsd, pl)
        ex, em = EO.pack(x.view(torch.int16).numpy(), tw.numpy(), ids.numpy(), rs)
        np.testing.assert_array_equal(x_send.view(torch.int16).cpu().numpy(), ex)
        np.testing.assert_array_equal(meta.cpu().numpy(), em)


def test_combine_bitexact(ep):
    M, world, H = 333, 4, 512
    rng = np.random.default_rng(0)
    tok_row = np.full((M, world), -1, dtype=np.int32)
    n = 0
    for m in range(M):
        for r in range(world):
            if rng.random() < 0.6:
                tok_row[m, r] = n
                n += 1
    back = O.round_bf16(rng.standard_normal((n, H)).astype(np.float32) * 4)
    dev = torch.device("cuda")
    back_t = torch.from_numpy(back).to(torch.bfloat16).to(dev)
    out = ep.combine(back_t, torch.from_numpy(tok_row.reshape(-1)).to(dev), M, world, H)
    ref = O.round_bf16(EO.combine(back, tok_row))
    np.testing.assert_array_equal(out.float().cpu().numpy(), ref)


@pytest.mark.parametrize("world,M", [(4, 600), (8, 64), (2, 3000)])
def test_emulated_expert_parallel_layer(ep, world, M):
    """All ranks' owner-side work on one GPU: plan one source batch for G
    destinations, run each destination's expert_map forward on its rows with
    only its experts' weights, combine -- equals the all-experts forward."""
    from kernels import w4a16_moe as K
    from kernels.synthetic import make_hidden, make_layer, make_routing

    E, H, I, k = 256, 3072, 1024, 10
    dev = torch.device("cuda")
    layer = make_layer(E, H, I, seed=0, device="cuda")
    w1r, s1r = K.repack_weights(layer["w1_q"], layer["w1_s"])
    w2r, s2r = K.repack_weights(layer["w2_q"], layer["w2_s"])
    del layer
    x = make_hidden(M, H, device="cuda")
    tw, ids = make_routing(M, E, k, device="cuda")
    full = K.fused_experts_w4a16(x, w1r, w2r, s1r, s2r, tw, ids)

    rc, ro, rs, rt = EO.plan(ids.cpu().numpy(), E, world)
    pl = ep.Plan(rc.tolist(), rc.tolist(), torch.from_numpy(ro).to(dev), torch.from_numpy(rs).to(dev),
                 torch.from_numpy(rt.reshape(-1)).to(dev))
    x_send, meta = ep.pack(x, tw, ids, pl)
    backs = []
    for r in range(world):
        rows = slice(int(ro[r]), int(ro[r + 1]))
        own = ep.owned_experts(E, world, r)
        y = K.fused_experts_w4a16(x_send[rows], w1r[own.start:own.stop], w2r[own.start:own.stop],
                                  s1r[own.start:own.stop], s2r[own.start:own.stop],
                                  meta[rows, k:].contiguous().view(torch.float32), meta[rows, :k].contiguous(),
                                  expert_map=ep.local_expert_map(E, world, r, dev), global_num_experts=E)
        backs.append(y)
    back = torch.cat(backs)
    out = ep.combine(back, pl.tok_row, M, world, H)
    d = ((out.float() - full.float()).norm() / full.float().norm()).item()
    assert d < 5e-3, d


@pytest.mark.parametrize("world,M", [(4, 600), (8, 64), (2, 3000), (1, 17)])
def test_emulated_fixed_capacity_layer(ep, world, M):
    """Fixed-capacity exchange, all ranks' work on one GPU: block r of the send
    buffer is what rank r receives from this source; its padding rows route
    nowhere; the combined result equals the all-experts forward."""
    from kernels import w4a16_moe as K
    from kernels.synthetic import make_hidden, make_layer, make_routing

    E, H, I, k = 256, 3072, 1024, 10
    dev = torch.device("cuda")
    layer = make_layer(E, H, I, seed=0, device="cuda")
    w1r, s1r = K.repack_weights(layer["w1_q"], layer["w1_s"])
    w2r, s2r = K.repack_weights(layer["w2_q"], layer["w2_s"])
    del layer
    x = make_hidden(M, H, device="cuda")
    tw, ids = make_routing(M, E, k, device="cuda")
    full = K.fused_experts_w4a16(x, w1r, w2r, s1r, s2r, tw, ids)
    cap = M + 5
    d = ep.dispatch_fixed(x, tw, ids, E, world, cap)
    rc, _, rs, rt = EO.plan(ids.cpu().numpy(), E, world)
    np.testing.assert_array_equal(d.counts.cpu().numpy(), rc)
    backs = []
    for r in range(world):
        blk = d.send[r * cap:(r + 1) * cap]
        xr, idr, wr = ep.unpack_rows(blk, H, k)
        assert (idr[int(rc[r]):] == -1).all()
        assert torch.equal(xr[: int(rc[r])], x[torch.as_tensor(rs[int(sum(rc[:r])):int(sum(rc[:r + 1]))],
                                                              device=dev, dtype=torch.int64)])
        own = ep.owned_experts(E, world, r)
        backs.append(K.fused_experts_w4a16(xr, w1r[own.start:own.stop], w2r[own.start:own.stop],
                                           s1r[own.start:own.stop], s2r[own.start:own.stop], wr, idr,
                                           expert_map=ep.local_expert_map(E, world, r, dev), global_num_experts=E))
    out = ep.combine(torch.cat(backs), d.tok_row, M, world, H)
    dd = ((out.float() - full.float()).norm() / full.float().norm()).item()
    assert dd < 5e-3, dd


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nccl_two_ranks():
    import torch.multiprocessing as mp

    import ep_worker

    cfg = dict(E=256, H=3072, I=1024, M=512, topk=10, seed=1)
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(ep_worker.gpu_rank, args=(2, _free_port(), cfg, d), nprocs=2, join=True)
        res = [Path(d, f"rank{r}.txt").read_text().split() for r in range(2)]
    assert all(r[0] == "1" for r in res), res
