"""Expert-parallel W4A16 MoE layers over ``torch.distributed`` (NCCL on GPUs).

The reference runs one GPU and has no expert parallelism; vLLM's EP contract
(``expert_map`` / ``global_num_experts`` in ``apply()``,
compressed_tensors_moe_wna16.py) is what :func:`fused_experts_w4a16` accepts,
and this module builds the token exchange around it:

* rank ``r`` of ``G`` owns experts ``[r*E/G, (r+1)*E/G)`` and only their
  repacked weights;
* each source token is sent once to every rank that owns one of its top-k
  experts (deduplicated per rank, not per slot), with its top-k ids and
  weights (:func:`plan`, ``w4a16_ep_plan`` / ``w4a16_ep_pack``);
* the owner runs :func:`fused_experts_w4a16` with its ``expert_map`` over the
  received rows -- slots of other ranks' experts contribute nothing -- and
  returns one bf16 row per (token, owner rank);
* the source sums those rows in rank order in fp32 (``w4a16_ep_combine``).

Collectives: one ``all_to_all_single`` of the per-rank counts (read back to the
host for the split sizes), then rows + routing metadata out and result rows
back.  :func:`exchange` is plain ``torch.distributed`` and runs on ``gloo``
ranks on CPU as well.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from kernels import w4a16_moe as _K

_BOUND = False


def _lib() -> ctypes.CDLL:
    global _BOUND
    lib = _K.load_library()
    if not _BOUND:
        c_i64, c_int, c_vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
        lib.w4a16_ep_plan.restype = c_int
        lib.w4a16_ep_plan.argtypes = [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp]
        lib.w4a16_ep_pack.restype = c_int
        lib.w4a16_ep_pack.argtypes = [c_vp, c_i64, c_vp, c_int, c_vp, c_i64, c_i64, c_i64, c_i64,
                                      c_vp, c_vp, c_vp, c_vp, c_vp]
        lib.w4a16_ep_dispatch_fixed.restype = c_int
        lib.w4a16_ep_dispatch_fixed.argtypes = [c_vp, c_i64, c_vp, c_int, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64,
                                                c_i64, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp]
        lib.w4a16_ep_combine.restype = c_int
        lib.w4a16_ep_combine.argtypes = [c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp]
        _BOUND = True
    return lib


def owned_experts(num_experts: int, world: int, rank: int) -> range:
    """Global ids of the experts rank ``rank`` owns (contiguous, E % G == 0)."""
    assert num_experts % world == 0, "experts must divide evenly over ranks"
    per = num_experts // world
    return range(rank * per, (rank + 1) * per)


def balanced_placement(load: torch.Tensor, world: int) -> torch.Tensor:
    """Expert placement balanced by measured load, as a relabelling.

    ``load[e]`` is how many routed slots expert ``e`` received on a
    calibration batch.  Returns ``perm`` (int64 [E]) with ``perm[e]`` the
    placed id of expert ``e``; rank r then owns the placed ids
    [r * E / G, (r + 1) * E / G) exactly as in :func:`owned_experts`, so the
    exchange kernels are unchanged.  A deployment applies it once at load
    time: permute the router's output rows (the router then emits placed ids)
    and store expert ``e``'s weights at position ``perm[e]``.

    Greedy and deterministic: experts in descending load (ties: lower id) go
    to the rank with the smallest total so far among ranks with a free slot
    (ties: lower rank); each rank takes exactly E / G experts.
    """
    E = load.numel()
    assert E % world == 0, "experts must divide evenly over ranks"
    per = E // world
    ld = load.detach().to("cpu", torch.float64)
    order = sorted(range(E), key=lambda e: (-float(ld[e]), e))
    total = [0.0] * world
    fill = [0] * world
    perm = torch.empty(E, dtype=torch.int64)
    for e in order:
        r = min((x for x in range(world) if fill[x] < per), key=lambda x: (total[x], x))
        perm[e] = r * per + fill[r]
        fill[r] += 1
        total[r] += float(ld[e])
    return perm


def local_expert_map(num_experts: int, world: int, rank: int, device) -> torch.Tensor:
    """vLLM-style ``expert_map``: global id -> local id, or -1 if not owned."""
    emap = torch.full((num_experts,), -1, dtype=torch.int32)
    r = owned_experts(num_experts, world, rank)
    emap[r.start:r.stop] = torch.arange(len(r), dtype=torch.int32)
    return emap.to(device)


def exchange(send: torch.Tensor, send_counts: list[int], recv_counts: list[int], group=None) -> torch.Tensor:
    """All-to-all-v of rows: ``send`` holds ``send_counts[r]`` rows for rank r
    (rank-major); returns the rows received, ``recv_counts[r]`` from rank r."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return send[: send_counts[0]]
    recv = send.new_empty((sum(recv_counts),) + tuple(send.shape[1:]))
    dist.all_to_all_single(recv, send[: sum(send_counts)].contiguous(), recv_counts, send_counts, group=group)
    return recv


def exchange_counts(send_counts: torch.Tensor, group=None) -> torch.Tensor:
    """Counts each rank will receive from every rank (transpose of the send counts)."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return send_counts.clone()
    recv = torch.empty_like(send_counts)
    dist.all_to_all_single(recv, send_counts, group=group)
    return recv


@dataclass
class Plan:
    """Send layout of one source batch (device tensors + host split sizes)."""

    send_counts: list[int]
    recv_counts: list[int]
    offsets: torch.Tensor  # [G+1] int32, rank-major send order
    send_tok: torch.Tensor  # [M*G] int32, token of each send row
    tok_row: torch.Tensor  # [M*G] int32, send row of (token, rank) or -1


def plan(topk_ids: torch.Tensor, num_experts: int, group=None) -> Plan:
    """Destination ranks per token (GPU kernel), then the count exchange."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    M, topk = topk_ids.shape
    dev = topk_ids.device
    ids = topk_ids if topk_ids.dtype in (torch.int32, torch.int64) else topk_ids.to(torch.int32)
    ids = ids.contiguous()
    counts = torch.empty(world, dtype=torch.int32, device=dev)
    offsets = torch.empty(world + 1, dtype=torch.int32, device=dev)
    send_tok = torch.empty(max(M * world, 1), dtype=torch.int32, device=dev)
    tok_row = torch.empty(max(M * world, 1), dtype=torch.int32, device=dev)
    lib = _lib()
    with torch.cuda.device(dev):
        _K._check(
            lib.w4a16_ep_plan(ids.data_ptr(), 1 if ids.dtype == torch.int64 else 0, M, topk, num_experts, world,
                              counts.data_ptr(), offsets.data_ptr(), send_tok.data_ptr(), tok_row.data_ptr(),
                              _K._stream_ptr(dev)),
            "w4a16_ep_plan",
        )
    recv = exchange_counts(counts, group)
    return Plan(counts.tolist(), recv.tolist(), offsets, send_tok, tok_row)


def pack(hidden: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor, pl: Plan):
    """Rows and routing metadata in send order: (x_send [n,H] bf16, meta [n,2k] int32)."""
    M, H = hidden.shape
    topk = topk_ids.shape[1]
    world = len(pl.send_counts)
    n = sum(pl.send_counts)
    dev = hidden.device
    x_send = torch.empty((max(n, 1), H), dtype=torch.bfloat16, device=dev)
    meta = torch.empty((max(n, 1), 2 * topk), dtype=torch.int32, device=dev)
    ids = topk_ids if topk_ids.dtype in (torch.int32, torch.int64) else topk_ids.to(torch.int32)
    ids = ids.contiguous()
    tw = topk_weights.to(torch.float32).contiguous()
    if hidden.stride(1) != 1:
        hidden = hidden.contiguous()
    with torch.cuda.device(dev):
        _K._check(
            _lib().w4a16_ep_pack(hidden.data_ptr(), hidden.stride(0), ids.data_ptr(),
                                 1 if ids.dtype == torch.int64 else 0, tw.data_ptr(), M, topk, H, world,
                                 pl.offsets.data_ptr(), pl.send_tok.data_ptr(), x_send.data_ptr(), meta.data_ptr(),
                                 _K._stream_ptr(dev)),
            "w4a16_ep_pack",
        )
    return x_send[:n], meta[:n]


def combine(back: torch.Tensor, tok_row: torch.Tensor, M: int, world: int, H: int) -> torch.Tensor:
    """out[m] = bf16(sum over owner ranks, in rank order, of the returned rows)."""
    out = torch.empty((M, H), dtype=torch.bfloat16, device=tok_row.device)
    if M == 0:
        return out
    if back.shape[0] == 0:  # nothing was sent anywhere: every row is zero
        back = out.new_zeros((1, H))
    with torch.cuda.device(out.device):
        _K._check(
            _lib().w4a16_ep_combine(back.data_ptr(), tok_row.data_ptr(), M, world, H, out.data_ptr(),
                                    _K._stream_ptr(out.device)),
            "w4a16_ep_combine",
        )
    return out


@dataclass
class LocalExperts:
    """This rank's repacked weights of one layer (experts owned_experts(E, G, rank))."""

    w13: torch.Tensor
    s13: torch.Tensor
    w2: torch.Tensor
    s2: torch.Tensor


EP_STAGES = ("plan+counts", "pack", "dispatch", "experts", "return", "combine")


def row_stride(H: int, topk: int) -> int:
    """bf16 elements per fixed-capacity send row: hidden, then 2*topk int32 of routing."""
    return H + (4 * topk + 7) // 8 * 8


@dataclass
class FixedDispatch:
    """Send blocks of the fixed-capacity exchange (device tensors only)."""

    send: torch.Tensor  # [G * capacity, row_stride] bf16
    counts: torch.Tensor  # [G] int32 valid rows per block
    send_tok: torch.Tensor  # [G * capacity] int32
    tok_row: torch.Tensor  # [M * G] int32, returned row of (token, rank) or -1
    capacity: int


def dispatch_fixed(hidden: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor, num_experts: int,
                   world: int, capacity: int) -> FixedDispatch:
    """Plan + pack into ``world`` blocks of ``capacity`` rows (one GPU kernel
    pair, no host synchronisation); routing metadata rides in each row."""
    M, H = hidden.shape
    topk = topk_ids.shape[1]
    dev = hidden.device
    rs = row_stride(H, topk)
    ids = topk_ids if topk_ids.dtype in (torch.int32, torch.int64) else topk_ids.to(torch.int32)
    ids = ids.contiguous()
    tw = topk_weights.to(torch.float32).contiguous()
    if hidden.stride(1) != 1:
        hidden = hidden.contiguous()
    send = torch.empty((world * capacity, rs), dtype=torch.bfloat16, device=dev)
    counts = torch.empty(world * (1 + (M + 1023) // 1024), dtype=torch.int32, device=dev)
    send_tok = torch.empty(max(world * capacity, 1), dtype=torch.int32, device=dev)
    tok_row = torch.empty(max(M * world, 1), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _K._check(
            _lib().w4a16_ep_dispatch_fixed(hidden.data_ptr(), hidden.stride(0), ids.data_ptr(),
                                           1 if ids.dtype == torch.int64 else 0, tw.data_ptr(), M, topk,
                                           num_experts, H, world, capacity, rs, send.data_ptr(), counts.data_ptr(),
                                           send_tok.data_ptr(), tok_row.data_ptr(), _K._stream_ptr(dev)),
            "w4a16_ep_dispatch_fixed",
        )
    return FixedDispatch(send, counts[:world], send_tok, tok_row, capacity)


def unpack_rows(rows: torch.Tensor, H: int, topk: int):
    """(hidden view [N, H] with row stride, ids [N, topk] int32, weights [N, topk] fp32) of received rows."""
    ids = rows[:, H:H + 2 * topk].contiguous().view(torch.int32)
    w = rows[:, H + 2 * topk:H + 4 * topk].contiguous().view(torch.float32)
    return rows[:, :H], ids, w


def all_to_all_equal(x: torch.Tensor, group=None) -> torch.Tensor:
    """All-to-all with equal splits (block r of x goes to rank r)."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return x
    out = torch.empty_like(x)
    dist.all_to_all_single(out, x, group=group)
    return out


def moe_layer(hidden: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor, experts: LocalExperts,
              num_experts: int, expert_map: torch.Tensor, group=None, stage_events=None,
              capacity: int | None = None) -> torch.Tensor:
    """One expert-parallel MoE layer for this rank's source tokens.

    ``topk_ids`` hold global expert ids.  Returns ``[M, H]`` bf16: the same
    result as a single-GPU :func:`fused_experts_w4a16` over all experts, up to
    the bf16 rounding of each owner rank's partial sum.  ``stage_events``
    (optional, profiling): a list of ``len(EP_STAGES) + 1`` CUDA events recorded
    on the current stream at the stage boundaries (plan and count exchange
    with its host read, pack, row dispatch, local experts, row return,
    combine).  ``capacity`` (>= M, equal on every rank) selects the
    fixed-capacity exchange: :func:`dispatch_fixed`, one all-to-all of rows
    with their routing each way, no host synchronisation.
    """
    ev = stage_events

    def mark(i):
        if ev is not None:
            ev[i].record()

    M, H = hidden.shape
    if capacity is not None:
        return _moe_layer_fixed(hidden, topk_weights, topk_ids, experts, num_experts, expert_map, group, mark,
                                capacity)
    mark(0)
    pl = plan(topk_ids, num_experts, group)
    mark(1)
    x_send, meta_send = pack(hidden, topk_weights, topk_ids, pl)
    mark(2)
    x_recv = exchange(x_send, pl.send_counts, pl.recv_counts, group)
    meta_recv = exchange(meta_send, pl.send_counts, pl.recv_counts, group)
    mark(3)
    topk = topk_ids.shape[1]
    if x_recv.shape[0] > 0:
        ids_recv = meta_recv[:, :topk].contiguous()
        w_recv = meta_recv[:, topk:].contiguous().view(torch.float32)
        y = _K.fused_experts_w4a16(x_recv, experts.w13, experts.w2, experts.s13, experts.s2, w_recv, ids_recv,
                                   expert_map=expert_map, global_num_experts=num_experts)
    else:
        y = x_recv.new_empty((0, H))
    mark(4)
    back = exchange(y, pl.recv_counts, pl.send_counts, group)
    mark(5)
    out = combine(back, pl.tok_row, M, len(pl.send_counts), H)
    mark(6)
    return out


def _moe_layer_fixed(hidden, topk_weights, topk_ids, experts, num_experts, expert_map, group, mark, capacity):
    M, H = hidden.shape
    topk = topk_ids.shape[1]
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    mark(0)
    d = dispatch_fixed(hidden, topk_weights, topk_ids, num_experts, world, capacity)
    mark(1)
    mark(2)
    recv = all_to_all_equal(d.send, group)
    mark(3)
    x_recv, ids_recv, w_recv = unpack_rows(recv, H, topk)
    y = _K.fused_experts_w4a16(x_recv, experts.w13, experts.w2, experts.s13, experts.s2, w_recv, ids_recv,
                               expert_map=expert_map, global_num_experts=num_experts)
    mark(4)
    back = all_to_all_equal(y, group)
    mark(5)
    out = combine(back, d.tok_row, M, world, H)
    mark(6)
    return out
