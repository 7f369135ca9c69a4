"""Expert-parallel exchange on CPU: the oracle planner's invariants, and the
product's collective layer (kernels.ep.exchange / exchange_counts) driven by
2 and 4 gloo ranks around the oracle's plan / pack / expert compute / combine,
checked against the single-process fp32 reference."""

from __future__ import annotations

import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import ep_oracle as EO


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_invariants(world):
    rng = np.random.default_rng(world)
    M, E, k = 97, 64, 6
    ids = np.stack([rng.choice(E, size=k, replace=False) for _ in range(M)]).astype(np.int32)
    counts, offsets, send_tok, tok_row = EO.plan(ids, E, world)
    owners = EO.owner_of(ids, E, world)
    for m in range(M):
        dest = sorted(set(owners[m].tolist()))
        assert [r for r in range(world) if tok_row[m, r] >= 0] == dest  # once per owner rank
        for r in dest:
            assert send_tok[tok_row[m, r]] == m
            assert offsets[r] <= tok_row[m, r] < offsets[r + 1]
    for r in range(world):  # tokens ascending inside a rank's segment
        seg = send_tok[offsets[r]:offsets[r + 1]]
        assert np.all(np.diff(seg) > 0)
    assert counts.sum() == len(send_tok) == offsets[-1]


def test_plan_ignores_invalid_ids():
    ids = np.array([[0, -1], [7, 99]], dtype=np.int32)
    counts, offsets, send_tok, tok_row = EO.plan(ids, 8, 2)
    assert counts.tolist() == [1, 1]
    assert tok_row.tolist() == [[0, -1], [-1, 1]]


def test_combine_sums_in_rank_order():
    back = np.array([[1.0, 2.0], [10.0, 20.0], [100.0, 200.0]], dtype=np.float32)
    tok_row = np.array([[0, 2], [-1, 1], [-1, -1]], dtype=np.int32)
    out = EO.combine(back, tok_row)
    np.testing.assert_array_equal(out, [[101.0, 202.0], [10.0, 20.0], [0.0, 0.0]])


@pytest.mark.parametrize("world", [2, 4])
def test_exchange_gloo_end_to_end(world):
    import ep_worker

    cfg = dict(E=8, H=256, I=128, M=24, topk=2, seed=3)
    mp.spawn(ep_worker.cpu_rank, args=(world, _free_port(), cfg), nprocs=world, join=True)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_balanced_placement_is_a_balanced_relabelling(world):
    """balanced_placement returns a permutation giving every rank E / G
    experts, is deterministic, and on the benchmark's Zipf routing it lowers
    the busiest rank's load below the contiguous split's on a held-out batch."""
    import torch

    from kernels import ep
    from kernels.synthetic import make_routing, zipf_bias

    E, topk = 256, 10
    bias = zipf_bias(E, 1.1, seed=0)
    _, calib = make_routing(8192, E, topk, seed=424_242, bias=bias)
    load = torch.bincount(calib.flatten().long(), minlength=E)
    perm = ep.balanced_placement(load, world)
    assert torch.equal(torch.sort(perm).values, torch.arange(E))
    assert torch.equal(perm, ep.balanced_placement(load, world))
    per = E // world
    assert all(int(((perm // per) == r).sum()) == per for r in range(world))

    _, test_ids = make_routing(8192, E, topk, seed=7, bias=bias)
    c = torch.bincount(test_ids.flatten().long(), minlength=E).double()
    contiguous = max(float(c[r * per:(r + 1) * per].sum()) for r in range(world))
    placed = torch.zeros(world, dtype=torch.float64).index_add_(0, perm // per, c)
    assert float(placed.max()) < contiguous
