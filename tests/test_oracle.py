"""CPU: pin the numpy oracle against fixtures produced by the reference itself
(tests/golden/make_golden.py) and against the reference's recorded numbers."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O


def _cases(golden_dir):
    d = np.load(golden_dir / "align_cases.npz")
    names = sorted({k.split("__")[0] for k in d.files})
    return d, names


def test_align_matches_reference_fixtures(golden_dir):
    d, names = _cases(golden_dir)
    assert len(names) >= 10
    for name in names:
        M, topk, E, bs = (int(v) for v in d[f"{name}__meta"])
        s, e, n = O.align_block_size(d[f"{name}__ids"], bs, E)
        np.testing.assert_array_equal(s, d[f"{name}__sorted"], err_msg=name)
        np.testing.assert_array_equal(e, d[f"{name}__expert_ids"], err_msg=name)
        np.testing.assert_array_equal(n, d[f"{name}__num_post"], err_msg=name)
        assert s.size == O.align_buffer_len(M * topk, E, bs)


def test_align_invariants_random():
    rng = np.random.default_rng(0)
    for _ in range(20):
        M, k, E, bs = int(rng.integers(0, 300)), int(rng.integers(1, 9)), int(rng.integers(1, 70)), int(rng.choice([1, 4, 16, 64]))
        ids = rng.integers(0, E, size=(M, k))
        s, e, n = O.align_block_size(ids, bs, E)
        flat = ids.reshape(-1)
        valid = s[s < M * k]
        assert sorted(valid.tolist()) == list(range(M * k))  # permutation of slots
        assert n[0] % bs == 0
        # each block holds one expert's slots, ascending
        for b in range(n[0] // bs):
            blk = s[b * bs:(b + 1) * bs]
            blk = blk[blk < M * k]
            assert np.all(flat[blk] == e[b])
            assert np.all(np.diff(blk) > 0)
        assert np.all(e[n[0] // bs:] == -1)


def test_pack_and_dequant_match_reference(golden_dir):
    c = np.load(golden_dir / "config0.npz")
    assert bool(c["int32_view_equals_nibble_pack"])
    for w, s, ref in (("w1_q", "w1_s_bits", "ref_w1_dequant_bf16_bits_e01"),
                      ("w2_q", "w2_s_bits", "ref_w2_dequant_bf16_bits_e01")):
        codes = O.unpack_int4_nibbles(c[w])
        np.testing.assert_array_equal(O.pack_int4_nibbles(codes), c[w])
        got = O.f32_to_bf16_bits(O.dequant(c[w][:2], c[s][:2], 32, round_to_bf16=True))
        np.testing.assert_array_equal(got, c[ref])
    # compressed-tensors int32 form -> uint8 view == nibble pack
    codes = O.unpack_int4_nibbles(c["w1_q"])
    np.testing.assert_array_equal(O.int32_pack_to_uint8(O.pack_int32_along_k(codes)), c["w1_q"])


def test_moe_reference_matches_reference_run(golden_dir):
    c = np.load(golden_dir / "config0.npz")
    x = O.bf16_bits_to_f32(c["hidden_bits"])
    out = O.moe_reference(x, c["w1_q"], c["w1_s_bits"], c["w2_q"], c["w2_s_bits"],
                          c["topk_weights"], c["topk_ids"], 32)
    np.testing.assert_allclose(out, c["ref_out_fp32"], rtol=1e-5, atol=1e-5)
    out16 = O.moe_reference(x, c["w1_q"], c["w1_s_bits"], c["w2_q"], c["w2_s_bits"],
                            c["topk_weights"], c["topk_ids"], 32, round_weights_to_bf16=True)
    ref16 = O.bf16_bits_to_f32(c["ref_out_bf16_bits"])
    assert O.rel_frobenius(out16, ref16) < 5e-3
    assert O.max_abs_err(out16, c["ref_out_fp32"]) < 2e-2


def test_synthetic_config0_matches_fixture(golden_dir):
    from kernels.synthetic import config0

    c = np.load(golden_dir / "config0.npz")
    g = config0("cpu")
    np.testing.assert_array_equal(g["w1_q"].numpy(), c["w1_q"])
    np.testing.assert_array_equal(g["topk_ids"].numpy(), c["topk_ids"])
    np.testing.assert_array_equal(g["hidden"].view(torch.int16).numpy().view(np.uint16), c["hidden_bits"])


def test_routing_known_answers(golden_dir):
    """Unique experts / weight bytes of the reference's make_routing (recorded in
    its results/showdown2.json as 10/38/119/238/256) from our generator."""
    from kernels.synthetic import make_routing

    known = json.loads((golden_dir / "routing_known.json").read_text())
    assert [r["unique_experts"] for r in known["rows"]] == [10, 38, 119, 238, 256]
    for row in known["rows"]:
        tw, ids = make_routing(row["M"], 256, 10, seed=0)
        assert ids.reshape(-1)[:20].tolist() == row["ids_head"]
        np.testing.assert_allclose(tw.reshape(-1)[:10].numpy(), row["weights_head"], rtol=1e-6)
        n = int(torch.unique(ids).numel())
        assert n == row["unique_experts"]
        assert O.weight_bytes_for_experts(n, 3072, 1024, 32) == row["weight_bytes"]


def test_repack_layout_roundtrip():
    rng = np.random.default_rng(1)
    E, N, K = 2, 32, 128
    w_q = rng.integers(0, 256, size=(E, N, K // 2), dtype=np.uint8)
    s = rng.integers(0, 65535, size=(E, N, K // 32), dtype=np.uint16)
    w_rep, s_rep = O.repack_layout(w_q, s, 32)
    assert w_rep.shape == (E, N // 16, K // 64, 512) and s_rep.shape == (E, N // 16, K // 64, 32)
    codes = O.unpack_int4_nibbles(w_q)
    words = w_rep.view("<u4").reshape(E, N // 16, K // 64, 32, 4)
    for e, r, cc, lane, j, i in [(0, 0, 0, 0, 0, 0), (1, 1, 1, 31, 3, 7), (0, 1, 0, 13, 2, 5), (1, 0, 1, 6, 1, 2)]:
        g, t = lane >> 2, lane & 3
        row = r * 16 + g + 8 * (i & 1)
        k = cc * 64 + 16 * j + 2 * t + 8 * ((i >> 1) & 1) + (i >> 2)
        assert (int(words[e, r, cc, lane, j]) >> (4 * i)) & 0xF == codes[e, row, k]
    # every code appears exactly once
    assert np.sort(O.unpack_int4_nibbles(w_rep).reshape(-1)).tolist() == np.sort(codes.reshape(-1)).tolist()
    # scales: group 64 storage replicates
    w64, s64 = O.repack_layout(w_q, s[..., ::2].copy(), 64)
    assert s64[0, 0, 0, 0] == s[0, 0, 0] and s64[0, 0, 0, 2] == s[0, 0, 0]


def test_bf16_helpers():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.3, 0.0, 65504.0], dtype=np.float32)
    np.testing.assert_array_equal(O.round_bf16(x), torch.tensor(x).to(torch.bfloat16).float().numpy())
    y = np.random.default_rng(3).standard_normal(1000).astype(np.float32) * 100
    np.testing.assert_array_equal(O.f32_to_bf16_bits(y), torch.tensor(y).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))


@pytest.mark.parametrize("M", [1, 7])
def test_expert_map_reference_semantics(M):
    rng = np.random.default_rng(M)
    E, H, I, k = 4, 64, 64, 2
    w1 = rng.integers(0, 256, size=(E, 2 * I, H // 2), dtype=np.uint8)
    w2 = rng.integers(0, 256, size=(E, H, I // 2), dtype=np.uint8)
    s1 = O.f32_to_bf16_bits(rng.uniform(0.005, 0.02, size=(E, 2 * I, H // 32)).astype(np.float32))
    s2 = O.f32_to_bf16_bits(rng.uniform(0.005, 0.02, size=(E, H, I // 32)).astype(np.float32))
    x = O.round_bf16(rng.standard_normal((M, H)).astype(np.float32))
    ids = rng.integers(0, 8, size=(M, k))
    tw = rng.uniform(0, 1, size=(M, k)).astype(np.float32)
    emap = np.array([-1, 0, -1, 1, 2, -1, 3, -1])
    full = np.zeros((8, 2 * I, H // 2), np.uint8)
    out = O.moe_reference(x, w1, s1, w2, s2, tw, ids, 32, expert_map=emap)
    # same thing by remapping ids by hand
    local = np.where(emap[ids] >= 0, emap[ids], 99)
    out2 = O.moe_reference(x, w1, s1, w2, s2, tw, local, 32)
    np.testing.assert_allclose(out, out2, rtol=0, atol=0)
    del full
