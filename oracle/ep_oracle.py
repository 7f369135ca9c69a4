"""CPU oracle for the expert-parallel token exchange -- TEST INFRASTRUCTURE ONLY.

Plain numpy statements of what ``w4a16_ep_plan`` / ``w4a16_ep_pack`` /
``w4a16_ep_combine`` compute, used by ``tests/`` as the checker (the product
path never imports this module).  The reference has no expert parallelism
(it runs one GPU); the contract restated here is this library's, built on
vLLM's ``expert_map`` convention (global id -> local id or -1) that the
reference's call site drops (``integration/apply.py:158-167``).  The single-GPU
``moe_reference`` of ``oracle/moe_oracle.py`` is the end-to-end target: an
expert-parallel layer must equal it up to the bf16 rounding of each owner
rank's partial sum.
"""

from __future__ import annotations

import numpy as np


def owner_of(expert_ids: np.ndarray, num_experts: int, world: int) -> np.ndarray:
    """Rank owning each global expert id (contiguous blocks of E/G)."""
    return expert_ids // (num_experts // world)


def plan(topk_ids: np.ndarray, num_experts: int, world: int):
    """(counts [G], offsets [G+1], send_tok [n], tok_row [M, G]).

    Rank-major send order; inside a rank, tokens ascending; a token appears
    once per destination rank however many of its slots that rank owns.
    """
    M = topk_ids.shape[0]
    dest = np.zeros((M, world), dtype=bool)
    valid = (topk_ids >= 0) & (topk_ids < num_experts)
    owners = np.where(valid, owner_of(np.where(valid, topk_ids, 0), num_experts, world), -1)
    for r in range(world):
        dest[:, r] = (owners == r).any(axis=1)
    counts = dest.sum(axis=0).astype(np.int32)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    send_tok = np.concatenate([np.nonzero(dest[:, r])[0] for r in range(world)]).astype(np.int32)
    tok_row = np.full((M, world), -1, dtype=np.int32)
    for r in range(world):
        toks = np.nonzero(dest[:, r])[0]
        tok_row[toks, r] = offsets[r] + np.arange(len(toks))
    return counts, offsets, send_tok, tok_row


def pack(hidden: np.ndarray, topk_weights: np.ndarray, topk_ids: np.ndarray, send_tok: np.ndarray):
    """Rows and metadata in send order: meta = [ids int32 | weights fp32 bits]."""
    x_send = hidden[send_tok]
    ids = topk_ids[send_tok].astype(np.int32)
    wbits = topk_weights[send_tok].astype(np.float32).view(np.int32)
    return x_send, np.concatenate([ids, wbits], axis=1)


def combine(back_f32: np.ndarray, tok_row: np.ndarray) -> np.ndarray:
    """out[m] = sum over r ascending of back[tok_row[m, r]] (fp32), 0 if none."""
    M, world = tok_row.shape
    H = back_f32.shape[1] if back_f32.ndim == 2 else 0
    out = np.zeros((M, H), dtype=np.float32)
    for r in range(world):
        rows = tok_row[:, r]
        sel = rows >= 0
        out[sel] += back_f32[rows[sel]]
    return out


def local_expert_map(num_experts: int, world: int, rank: int) -> np.ndarray:
    per = num_experts // world
    emap = np.full(num_experts, -1, dtype=np.int32)
    emap[rank * per:(rank + 1) * per] = np.arange(per, dtype=np.int32)
    return emap
