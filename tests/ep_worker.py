"""Rank bodies for the multi-process expert-parallel tests (spawned by
``tests/test_ep_cpu.py`` on gloo and ``tests/test_ep_gpu.py`` on NCCL)."""

from __future__ import annotations

import os
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
for p in (str(REPO / "gb10-laguna-s-2.1-w4a16-moe_b200"), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def _init(rank: int, world: int, port: int, backend: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group(backend, rank=rank, world_size=world)


def small_problem(E: int, H: int, I: int, M: int, topk: int, seed: int):
    """Shared seeded problem: every rank builds the same arrays."""
    from kernels.synthetic import make_layer, make_routing

    layer = make_layer(E, H, I, seed=seed)
    g = torch.Generator().manual_seed(seed + 5)
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    tw, ids = make_routing(M, E, topk, seed=seed)
    return layer, x, tw, ids


def cpu_rank(rank: int, world: int, port: int, cfg: dict) -> None:
    """Oracle planner / packer / expert compute / combine around the product's
    collective layer (kernels.ep.exchange*), on gloo CPU ranks."""
    from kernels import ep
    from oracle import ep_oracle as EO
    from oracle import moe_oracle as O

    _init(rank, world, port, "gloo")
    try:
        E, H, I, M, topk = cfg["E"], cfg["H"], cfg["I"], cfg["M"], cfg["topk"]
        layer, x, tw, ids = small_problem(E, H, I, M, topk, cfg["seed"])
        lo, hi = rank * M // world, (rank + 1) * M // world  # this rank's source tokens
        xs = x[lo:hi].float().numpy()
        tws, idss = tw[lo:hi].numpy(), ids[lo:hi].numpy()
        w1q, w1s = layer["w1_q"].numpy(), layer["w1_s"].view(torch.int16).numpy().view(np.uint16)
        w2q, w2s = layer["w2_q"].numpy(), layer["w2_s"].view(torch.int16).numpy().view(np.uint16)

        counts, offsets, send_tok, tok_row = EO.plan(idss, E, world)
        recv_counts = ep.exchange_counts(torch.from_numpy(counts)).tolist()
        x_send, meta_send = EO.pack(xs, tws, idss, send_tok)
        x_recv = ep.exchange(torch.from_numpy(x_send), counts.tolist(), recv_counts).numpy()
        meta_recv = ep.exchange(torch.from_numpy(meta_send), counts.tolist(), recv_counts).numpy()
        ids_recv = meta_recv[:, :topk]
        w_recv = np.ascontiguousarray(meta_recv[:, topk:]).view(np.float32)
        own = ep.owned_experts(E, world, rank)
        emap = EO.local_expert_map(E, world, rank)
        y = O.moe_reference(x_recv, w1q[own.start:own.stop], w1s[own.start:own.stop], w2q[own.start:own.stop],
                            w2s[own.start:own.stop], w_recv, ids_recv, expert_map=emap)
        y = O.round_bf16(y)  # owner ranks return bf16 rows
        back = ep.exchange(torch.from_numpy(y), recv_counts, counts.tolist()).numpy()
        out = EO.combine(back, tok_row)

        ref = O.moe_reference(xs, w1q, w1s, w2q, w2s, tws, idss)
        err = O.rel_frobenius(out, ref)
        assert err < 5e-3, f"rank {rank}: rel Frobenius {err}"
        # every routed (token, rank) pair went out exactly once
        dests = {(int(m), int(EO.owner_of(e, E, world))) for m in range(hi - lo) for e in idss[m]}
        assert sum(counts) == len(dests)
    finally:
        dist.destroy_process_group()


def gpu_rank(rank: int, world: int, port: int, cfg: dict, result_dir: str) -> None:
    """Product path (plan / pack / NCCL all-to-all / forward / combine) on one
    GPU per rank, checked against a single-GPU forward over all experts."""
    from kernels import ep
    from kernels import w4a16_moe as K

    torch.cuda.set_device(rank)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    _init(rank, world, port, "nccl")
    try:
        E, H, I, M, topk = cfg["E"], cfg["H"], cfg["I"], cfg["M"], cfg["topk"]
        layer, x, tw, ids = small_problem(E, H, I, M, topk, cfg["seed"])
        dev = torch.device("cuda", rank)
        w1r, s1r = K.repack_weights(layer["w1_q"].to(dev), layer["w1_s"].to(dev))
        w2r, s2r = K.repack_weights(layer["w2_q"].to(dev), layer["w2_s"].to(dev))
        own = ep.owned_experts(E, world, rank)
        local = ep.LocalExperts(w1r[own.start:own.stop].contiguous(), s1r[own.start:own.stop].contiguous(),
                                w2r[own.start:own.stop].contiguous(), s2r[own.start:own.stop].contiguous())
        emap = ep.local_expert_map(E, world, rank, dev)
        lo, hi = rank * M // world, (rank + 1) * M // world
        xs, tws, idss = x[lo:hi].to(dev), tw[lo:hi].to(dev), ids[lo:hi].to(dev)
        out = ep.moe_layer(xs, tws, idss, local, E, emap)
        full = K.fused_experts_w4a16(xs, w1r, w2r, s1r, s2r, tws, idss)
        torch.cuda.synchronize()
        d = (out.float() - full.float()).norm() / full.float().norm().clamp_min(1e-30)
        ok = bool(d.item() < 5e-3)
        Path(result_dir, f"rank{rank}.txt").write_text(f"{int(ok)} {d.item():.3e}\n")
    finally:
        dist.destroy_process_group()
