"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no dataset or checkpoint is involved).

* Router: logits ~ N(0, 1) from a CPU ``torch.Generator`` seeded with
  ``seed + 17000 + M``, top-k of the logits, softmax over the k values.  This
  is the reference's ``make_routing`` (``bench/bench_moe.py:210-231``), which
  equals "softmax then top-k renormalised"; optional per-expert log-Zipf bias
  for the skewed expert-parallel configuration.
* Activations: bf16 ~ N(0, 1) (CPU generator, ``seed + 1000 + M``).
* Weights: stored int4 codes uniform in [0, 15] (q uniform in [-8, 7]) packed
  two per byte, generated directly on the target device; bf16 group scales
  uniform in [0.005, 0.02].
"""

from __future__ import annotations

import torch

# Layer shape of the benchmark configurations 1-4.
LAYER_E = 256
LAYER_TOPK = 10
LAYER_H = 3072
LAYER_I = 1024
GROUP = 32


def zipf_bias(E: int, s: float = 1.1, seed: int = 0) -> torch.Tensor:
    """bias_e = log(r_e^-s / sum_r r^-s), r_e = perm(seed)[e] + 1."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed + 23_000)
    perm = torch.randperm(E, generator=g)
    r = (perm + 1).to(torch.float64)
    p = r.pow(-s)
    return torch.log(p / p.sum()).to(torch.float32)


def make_routing(M: int, E: int, topk: int, seed: int = 0, device: str | torch.device = "cpu",
                 bias: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """(topk_weights [M, topk] fp32, topk_ids [M, topk] int32)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed + 17_000 + M)
    logits = torch.randn(M, E, generator=g, dtype=torch.float32)
    if bias is not None:
        logits = logits + bias.to(torch.float32)[None, :]
    vals, ids = torch.topk(logits, k=topk, dim=-1)
    weights = torch.softmax(vals, dim=-1)
    return weights.to(device), ids.to(device=device, dtype=torch.int32)


def make_hidden(M: int, H: int, seed: int = 0, device: str | torch.device = "cpu") -> torch.Tensor:
    g = torch.Generator(device="cpu")
    g.manual_seed(seed + 1000 + M)
    return torch.randn(M, H, generator=g).to(dtype=torch.bfloat16, device=device)


def make_packed_weights(E: int, N_out: int, K: int, group: int = GROUP, seed: int = 0,
                        device: str | torch.device = "cpu") -> tuple[torch.Tensor, torch.Tensor]:
    """(w_q (E, N_out, K/2) uint8, scales (E, N_out, K/group) bf16) on ``device``.

    Each byte is two independent uniform codes, i.e. a uniform byte.
    """
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    w_q = torch.randint(0, 256, (E, N_out, K // 2), generator=g, dtype=torch.uint8, device=dev)
    s = torch.empty((E, N_out, K // group), dtype=torch.float32, device=dev)
    s.uniform_(0.005, 0.02, generator=g)
    return w_q, s.to(torch.bfloat16)


def make_layer(E: int, H: int, I: int, group: int = GROUP, seed: int = 0,
               device: str | torch.device = "cpu") -> dict[str, torch.Tensor]:
    """Unpacked (vLLM post-load layout) w13 / w2 weights and scales of one layer."""
    w1_q, w1_s = make_packed_weights(E, 2 * I, H, group, seed=seed * 2 + 1, device=device)
    w2_q, w2_s = make_packed_weights(E, H, I, group, seed=seed * 2 + 2, device=device)
    return {"w1_q": w1_q, "w1_s": w1_s, "w2_q": w2_q, "w2_s": w2_s}


def config0(device: str | torch.device = "cpu") -> dict[str, torch.Tensor]:
    """Benchmark configuration 0: E=8, top-2, H=256, I=128, M=4, seed 0, with
    the weights in compressed-tensors int32 form (8 codes per int32 along K)
    converted to the vLLM uint8 view."""
    E, k, H, I, M = 8, 2, 256, 128, 4
    g = torch.Generator(device="cpu")
    g.manual_seed(0)
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(M, E, generator=g, dtype=torch.float32)
    probs = torch.softmax(logits, dim=-1)
    tw, ids = torch.topk(probs, k=k, dim=-1)
    tw = tw / tw.sum(dim=-1, keepdim=True)

    def packed(n_out: int, k_in: int):
        codes = torch.randint(0, 16, (E, n_out, k_in), generator=g, dtype=torch.int32)
        c = codes.reshape(E, n_out, k_in // 8, 8)
        word = torch.zeros(E, n_out, k_in // 8, dtype=torch.int64)
        for i in range(8):
            word |= c[..., i].to(torch.int64) << (4 * i)
        word = word.to(torch.int64)
        word = torch.where(word >= 2**31, word - 2**32, word).to(torch.int32)
        u8 = word.contiguous().view(torch.uint8).reshape(E, n_out, k_in // 2)
        s = (torch.rand(E, n_out, k_in // 32, generator=g) * 0.015 + 0.005).to(torch.bfloat16)
        return u8, s, codes

    w1_q, w1_s, c1 = packed(2 * I, H)
    w2_q, w2_s, c2 = packed(H, I)
    out = {"hidden": x, "topk_weights": tw.to(torch.float32), "topk_ids": ids.to(torch.int32),
           "w1_q": w1_q, "w1_s": w1_s, "w2_q": w2_q, "w2_s": w2_s,
           "w1_codes": c1.to(torch.uint8), "w2_codes": c2.to(torch.uint8)}
    return {k_: v.to(device) for k_, v in out.items()}
