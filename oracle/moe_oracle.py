"""CPU oracle for the W4A16 grouped-MoE hot path -- TEST INFRASTRUCTURE ONLY.

Plain numpy restatement of the reference algorithm, used by ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of ``bench.py`` as
the checker.  The product path (``kernels/w4a16_moe.py`` + the sm_100a
library) never imports this module.

Pinned against the reference itself: ``tests/golden/make_golden.py`` imports
the reference's own ``kernels/w4a16_moe.py`` and ``bench/bench_moe.py`` in a
container where they are mounted and stores their outputs under
``tests/golden/``; ``tests/test_oracle.py`` checks every function below
against those fixtures.

Functions and the reference code they restate (paths inside the reference):

* :func:`align_block_size`   -- ``kernels/w4a16_moe.py:141-290``
* :func:`pack_int4_nibbles`  -- ``bench/bench_moe.py:87-92``
* :func:`unpack_int4_nibbles`-- ``bench/bench_moe.py:95-99``
* :func:`dequant`            -- ``bench/bench_moe.py:102-119`` (fp32, or bf16-
                                rounded like the reference's dequant)
* :func:`moe_reference`      -- ``bench/bench_moe.py:271-303`` (run_reference +
                                silu_and_mul), fp32 accumulate
* :func:`weight_bytes_for_experts` -- ``bench/bench_moe.py:250-263``
* :func:`rel_frobenius`, :func:`max_abs_err` -- ``bench/bench_moe.py:520-527``
* :func:`repack_layout`      -- this library's own fragment-major layout
                                (no reference counterpart; the reference's
                                ``repack_weights`` layout is private to its
                                Triton kernels, ``tasks/TASK-03-kernel.md``)
"""

from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# bf16 helpers (bf16 values are carried as uint16 bit patterns)
# ---------------------------------------------------------------------------


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit pattern (NaN-preserving)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    r = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r = r.copy()
        r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest-even bf16 value, kept as fp32 (same result as
    ``bf16_bits_to_f32(f32_to_bf16_bits(x))``, in 32-bit arithmetic: for
    every non-NaN input the sum below stays under 2**32)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    r = (u >> 16) & np.uint32(1)
    r += np.uint32(0x7FFF)
    r += u
    r &= np.uint32(0xFFFF0000)
    out = r.view(np.float32)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.float32(np.nan)
    return out


# ---------------------------------------------------------------------------
# Routing: moe_align_block_size
# ---------------------------------------------------------------------------


def align_buffer_len(n_tok: int, num_experts: int, block_size: int) -> int:
    """reference kernels/w4a16_moe.py:153-156."""
    p = n_tok + num_experts * (block_size - 1)
    return (p + block_size - 1) // block_size * block_size


def align_block_size(topk_ids: np.ndarray, block_size: int, num_experts: int):
    """Expert-sorted, block-padded slot order (reference :187-290).

    Returns (sorted_token_ids[P] int32, expert_ids[P//bs] int32,
    num_tokens_post_padded[1] int32).  Within an expert the slot ids are in
    ascending order (the reference's stable sort, :263-278); padding holds
    ``n_tok``; blocks past ``num_post`` get expert -1.
    """
    ids = np.asarray(topk_ids).reshape(-1).astype(np.int64)
    n_tok = ids.size
    P = align_buffer_len(n_tok, num_experts, block_size)
    sorted_ids = np.full(P, n_tok, dtype=np.int32)
    expert_ids = np.full(P // block_size, -1, dtype=np.int32)
    if n_tok == 0:
        return sorted_ids, expert_ids, np.zeros(1, dtype=np.int32)
    counts = np.bincount(ids, minlength=num_experts)[:num_experts]
    padded = (counts + block_size - 1) // block_size * block_size
    offsets = np.zeros(num_experts + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(padded)
    order = np.argsort(ids, kind="stable")
    sorted_e = ids[order]
    first = np.searchsorted(sorted_e, np.arange(num_experts), side="left")
    rank = np.arange(n_tok) - first[sorted_e]
    sorted_ids[offsets[sorted_e] + rank] = order.astype(np.int32)
    block_tok0 = np.arange(P // block_size, dtype=np.int64) * block_size
    e_for_block = np.searchsorted(offsets[1:], block_tok0, side="right")
    valid = block_tok0 < offsets[-1]
    expert_ids[valid] = e_for_block[valid].astype(np.int32)
    return sorted_ids, expert_ids, np.array([offsets[-1]], dtype=np.int32)


# ---------------------------------------------------------------------------
# int4 packing / dequant
# ---------------------------------------------------------------------------


def pack_int4_nibbles(codes_u4: np.ndarray) -> np.ndarray:
    """Stored codes (q+8 in [0,15]) -> bytes, low nibble = even k."""
    c = np.asarray(codes_u4, dtype=np.uint8)
    assert c.shape[-1] % 2 == 0
    return (c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8)


def unpack_int4_nibbles(packed: np.ndarray) -> np.ndarray:
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = p & 0xF
    out[..., 1::2] = p >> 4
    return out


def pack_int32_along_k(codes_u4: np.ndarray) -> np.ndarray:
    """compressed-tensors ``pack-quantized``: 8 stored codes per int32 along K,
    code i at bits 4i (SP/compressed_tensors/.../pack_quantized/helpers.py)."""
    c = np.asarray(codes_u4, dtype=np.uint32)
    assert c.shape[-1] % 8 == 0
    c = c.reshape(c.shape[:-1] + (c.shape[-1] // 8, 8))
    word = np.zeros(c.shape[:-1], dtype=np.uint32)
    for i in range(8):
        word |= c[..., i] << (4 * i)
    return word.view(np.int32)


def int32_pack_to_uint8(packed_i32: np.ndarray) -> np.ndarray:
    """vLLM's post-load view: (E, N_out, K/8) int32 -> (E, N_out, K/2) uint8
    (little-endian; SP/vllm/.../compressed_tensors_moe_wna16.py:184-191)."""
    a = np.ascontiguousarray(packed_i32, dtype=np.int32)
    return a.view(np.uint8).reshape(a.shape[:-1] + (a.shape[-1] * 4,))


def dequant(packed: np.ndarray, scales_bits: np.ndarray, group_size: int,
            round_to_bf16: bool = False) -> np.ndarray:
    """(q - 8) * s with q from the packed bytes and s from bf16 bits.

    ``round_to_bf16=False`` keeps the product in fp32 (the fp32 reference);
    ``True`` rounds it to bf16 like the reference's dequant_int4_w4a16.
    """
    q = unpack_int4_nibbles(packed).astype(np.float32) - 8.0
    s = bf16_bits_to_f32(scales_bits)
    k = q.shape[-1]
    assert k % group_size == 0 and s.shape[-1] == k // group_size
    w = q * np.repeat(s, group_size, axis=-1)
    return round_bf16(w) if round_to_bf16 else w


# ---------------------------------------------------------------------------
# MoE layer
# ---------------------------------------------------------------------------


def silu(x: np.ndarray) -> np.ndarray:
    return x / (1.0 + np.exp(-x))


def moe_reference(hidden: np.ndarray, w1_q: np.ndarray, w1_s: np.ndarray, w2_q: np.ndarray,
                  w2_s: np.ndarray, topk_weights: np.ndarray, topk_ids: np.ndarray,
                  group_size: int = 32, expert_map: np.ndarray | None = None,
                  round_weights_to_bf16: bool = False,
                  round_intermediate_to_bf16: bool = False) -> np.ndarray:
    """fp32 per-expert reference of the fused MoE (bench/bench_moe.py:277-303).

    hidden: [M, H] fp32 values (already bf16-representable).
    w1_q (E, 2I, H/2) u8, w1_s (E, 2I, H/g) bf16 bits; w2_q (E, H, I/2),
    w2_s (E, H, I/g).  Returns fp32 [M, H]:
    out[m] = sum_t w[m,t] * W2_e(silu(W_gate,e x) * W_up,e x).
    With ``expert_map`` ids are global and mapped to local experts; -1 skips.
    ``round_weights_to_bf16`` rounds each dequantised weight to bf16 (the
    reference's ``dequant_int4_w4a16``, bench/bench_moe.py:119);
    ``round_intermediate_to_bf16`` rounds silu(gate)*up to bf16 before the w2
    product (the bf16 intermediate cache of vLLM's fused_experts and of the
    reference's kernel, kernels/w4a16_moe.py).
    """
    return moe_reference_variants(hidden, w1_q, w1_s, w2_q, w2_s, topk_weights, topk_ids, group_size,
                                  expert_map, [(round_weights_to_bf16, round_intermediate_to_bf16)])[0]


def moe_reference_variants(hidden, w1_q, w1_s, w2_q, w2_s, topk_weights, topk_ids, group_size=32,
                           expert_map=None, variants=((False, False),)):
    """:func:`moe_reference` for several (round_weights, round_intermediate)
    numerics at once, sharing the per-expert dequantisation."""
    M, H = hidden.shape
    outs = [np.zeros((M, H), dtype=np.float32) for _ in variants]
    ids = np.asarray(topk_ids).astype(np.int64)
    if expert_map is not None:
        emap = np.asarray(expert_map).astype(np.int64)
        ids = np.where((ids >= 0) & (ids < emap.size), emap[np.clip(ids, 0, emap.size - 1)], -1)
    tw = np.asarray(topk_weights, dtype=np.float32)
    h = np.asarray(hidden, dtype=np.float32)
    E = w1_q.shape[0]
    for e in range(E):
        tok, slot = np.nonzero(ids == e)
        if tok.size == 0:
            continue
        w1x = dequant(w1_q[e], w1_s[e], group_size, False)
        w2x = dequant(w2_q[e], w2_s[e], group_size, False)
        w1r = w2r = None
        for out, (rw, ri) in zip(outs, variants):
            if rw and w1r is None:
                w1r, w2r = round_bf16(w1x), round_bf16(w2x)
            w1, w2 = (w1r, w2r) if rw else (w1x, w2x)
            y = h[tok] @ w1.T
            d = y.shape[-1] // 2
            y = silu(y[:, :d]) * y[:, d:]
            if ri:
                y = round_bf16(y)
            y = y @ w2.T
            np.add.at(out, tok, y * tw[tok, slot][:, None])
    return outs


def weight_bytes_for_experts(n_experts: int, K: int, N: int, group_size: int) -> int:
    """Bytes of packed w13 + w2 + bf16 scales for n_experts (bench_moe.py:250-263)."""
    w1 = n_experts * (2 * N) * (K // 2)
    w2 = n_experts * K * (N // 2)
    s1 = n_experts * (2 * N) * (K // group_size) * 2
    s2 = n_experts * K * (N // group_size) * 2
    return w1 + w2 + s1 + s2


def rel_frobenius(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-12))


def max_abs_err(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def bf16_half_ulp(x: np.ndarray) -> np.ndarray:
    """Half a bf16 ulp at |x| (rounding bound of a bf16 output)."""
    ax = np.abs(np.asarray(x, dtype=np.float32))
    e = np.floor(np.log2(np.maximum(ax, np.float32(1e-30))))
    return np.ldexp(np.float32(1.0), (e - 8).astype(np.int32))


# ---------------------------------------------------------------------------
# This library's repacked layout (for bit-exact checks of the GPU repack)
# ---------------------------------------------------------------------------


def repack_layout(w_q: np.ndarray, scales_bits: np.ndarray, group_size: int):
    """Fragment-major layout: (E, N/16, K/64, 512) u8 and (E, N/16, K/64, 32) u16.

    Lane l (g=l>>2, t=l&3) of a (rowtile, chunk) block owns bytes [16l, 16l+16)
    = four little-endian words j; word j nibble i holds the code of
    (row, k) = (g + 8*(i&1), k0 + 2t + 8*((i>>1)&1) + (i>>2)), k0 = 64c + 16j.
    Scales: entry 4g+w = s(g + 8*(w&1), group 2c + (w>>1)).
    """
    E, N, Kh = w_q.shape
    K = Kh * 2
    assert N % 16 == 0 and K % 64 == 0 and group_size % 32 == 0
    codes = unpack_int4_nibbles(w_q).astype(np.uint32)  # (E, N, K)
    R, C = N // 16, K // 64
    c5 = codes.reshape(E, R, 16, C, 64)  # e, r, row16, c, k64
    words = np.zeros((E, R, C, 32, 4), dtype=np.uint32)
    lanes = np.arange(32)
    g, t = lanes >> 2, lanes & 3
    for j in range(4):
        for i in range(8):
            row = g + 8 * (i & 1)
            kk = 16 * j + 2 * t + 8 * ((i >> 1) & 1) + (i >> 2)
            val = c5[:, :, row, :, kk]  # advanced indices first: (32, E, R, C)
            words[:, :, :, :, j] |= np.moveaxis(val, 0, -1) << (4 * i)
    w_rep = words.astype("<u4").view(np.uint8).reshape(E, R, C, 512)
    s = np.asarray(scales_bits, dtype=np.uint16)
    s32 = np.repeat(s, group_size // 32, axis=-1)  # (E, N, K/32)
    s5 = s32.reshape(E, R, 16, C, 2)
    s_rep = np.zeros((E, R, C, 32), dtype=np.uint16)
    for gg in range(8):
        for w in range(4):
            s_rep[:, :, :, 4 * gg + w] = s5[:, :, gg + 8 * (w & 1), :, w >> 1]
    return w_rep, s_rep
