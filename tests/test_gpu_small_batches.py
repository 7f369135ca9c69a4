"""GPU parity of the fused decode path at the smallest batches (M <= 4
tokens) against the CPU oracle, through the C ABI, on the 256-expert / top-10
/ 3072 x 1024 layer and on edge cases of its routing (duplicate experts in a
token, int64 ids, strided rows, topk = 1 and 16, a shard with no local slot),
with the multi-kernel general path as a second opinion."""

from __future__ import annotations

import pytest
import torch

from test_gpu_parity import K, big_layer, check_close, oracle_for  # noqa: F401  (fixtures)

pytestmark = pytest.mark.gpu


@pytest.fixture
def lib_(K):  # noqa: F811
    """The library on its default path (the fused decode kernel at these M)."""
    K.set_path("auto")
    yield K


def _run(K, layer, hidden, tw, ids, **kw):  # noqa: F811
    return K.fused_experts_w4a16(hidden, layer["w1r"], layer["w2r"], layer["s1r"], layer["s2r"], tw, ids, **kw)


@pytest.mark.parametrize("M", [1, 2, 3, 4])
def test_small_matches_oracle(lib_, big_layer, M):  # noqa: F811
    from kernels.synthetic import make_hidden, make_routing

    hidden = make_hidden(M, 3072, device="cuda")
    tw, ids = make_routing(M, 256, 10, device="cuda")
    out = _run(lib_, big_layer, hidden, tw, ids)
    torch.cuda.synchronize()
    assert lib_.read_status((M, 3072), 10, 256, 1024) == 0
    check_close(out, oracle_for(hidden, big_layer, tw, ids), None, f"small M={M}")
    # counters and flags were left clean: a second and third call agree bit for bit
    for _ in range(2):
        assert torch.equal(_run(lib_, big_layer, hidden, tw, ids), out)


def test_small_duplicates_int64_strided(lib_, big_layer):  # noqa: F811
    from kernels.synthetic import make_hidden, make_routing

    M = 4
    base = make_hidden(M, 3072 + 64, device="cuda")
    hidden = base[:, :3072]
    tw, ids = make_routing(M, 256, 10, device="cuda")
    ids[0, 1] = ids[0, 0]       # one expert twice in a token
    ids[2, :] = 17              # all ten slots of a token on one expert
    ids[3, 4] = ids[1, 4]       # an expert shared by two tokens
    out = _run(lib_, big_layer, hidden, tw, ids.to(torch.int64))
    torch.cuda.synchronize()
    assert lib_.read_status((M, 3072), 10, 256, 1024) == 0
    check_close(out, oracle_for(hidden, big_layer, tw, ids), None, "small dups+int64+strided")


@pytest.mark.parametrize("M,topk", [(1, 1), (4, 1), (2, 16), (4, 16)])
def test_small_topk_variants(lib_, big_layer, M, topk):  # noqa: F811
    from kernels.synthetic import make_hidden, make_routing

    hidden = make_hidden(M, 3072, device="cuda")
    tw, ids = make_routing(M, 256, topk, device="cuda")
    out = _run(lib_, big_layer, hidden, tw, ids)
    torch.cuda.synchronize()
    check_close(out, oracle_for(hidden, big_layer, tw, ids), None, f"small M={M} topk={topk}")


def test_small_deterministic_and_token_permutation(lib_, big_layer):  # noqa: F811
    from kernels.synthetic import make_hidden, make_routing

    M = 4
    hidden = make_hidden(M, 3072, device="cuda")
    tw, ids = make_routing(M, 256, 10, device="cuda")
    a = _run(lib_, big_layer, hidden, tw, ids)
    b = _run(lib_, big_layer, hidden, tw, ids)
    assert torch.equal(a, b)
    perm = torch.tensor([2, 0, 3, 1], device="cuda")
    c = _run(lib_, big_layer, hidden[perm].contiguous(), tw[perm].contiguous(), ids[perm].contiguous())
    assert torch.equal(c, a[perm])


def test_small_expert_map(lib_, big_layer):  # noqa: F811
    """A 4-way expert shard: every shard matches the oracle on its experts, a
    shard no token routes to returns zeros, and the shards sum to the layer."""
    from kernels.synthetic import make_hidden, make_routing

    M = 3
    hidden = make_hidden(M, 3072, device="cuda")
    tw, ids = make_routing(M, 256, 10, device="cuda")
    ids[:, :] = torch.randint(0, 192, (M, 10), generator=torch.Generator().manual_seed(3)).cuda().int()
    total = torch.zeros(M, 3072, dtype=torch.float32, device="cuda")
    for r in range(4):
        emap = torch.full((256,), -1, dtype=torch.int32)
        emap[r * 64:(r + 1) * 64] = torch.arange(64, dtype=torch.int32)
        emap = emap.cuda()
        sl = slice(r * 64, (r + 1) * 64)
        loc = {k: big_layer[k][sl] for k in ("w1r", "s1r", "w2r", "s2r")}
        out = lib_.fused_experts_w4a16(hidden, loc["w1r"], loc["w2r"], loc["s1r"], loc["s2r"], tw, ids,
                                         expert_map=emap, global_num_experts=256)
        torch.cuda.synchronize()
        if r == 3:
            assert torch.count_nonzero(out) == 0
        else:
            sub = {"w1_q": big_layer["w1_q"][sl], "w1_s": big_layer["w1_s"][sl],
                   "w2_q": big_layer["w2_q"][sl], "w2_s": big_layer["w2_s"][sl]}
            check_close(out, oracle_for(hidden, sub, tw, ids, expert_map=emap), None, f"small shard {r}")
        total += out.float()
    # three bf16-rounded shard outputs summed and rounded again: up to ~2 ulp
    # from the one-pass reference, so the element count gets a stated bound
    check_close(total.to(torch.bfloat16), oracle_for(hidden, big_layer, tw, ids), None, "small shards summed", 2e-2)


def test_fused_agrees_with_general(K, big_layer):  # noqa: F811
    """The fused decode kernel and the multi-kernel general path, same inputs:
    within the parity tolerance of each other."""
    from kernels.synthetic import make_hidden, make_routing

    M = 2
    hidden = make_hidden(M, 3072, device="cuda")
    tw, ids = make_routing(M, 256, 10, device="cuda")
    K.set_path("auto")
    a = _run(K, big_layer, hidden, tw, ids)
    K.set_path("general")
    b = _run(K, big_layer, hidden, tw, ids)
    K.set_path("auto")
    torch.cuda.synchronize()
    # the two paths differ in weight numerics (exact (q - 8) vs bf16 (q - 8) * s),
    # so only the norm-wise forms apply between them
    check_close(a, b.float().cpu().numpy(), None, "fused vs general", outside_tol=1.0)
