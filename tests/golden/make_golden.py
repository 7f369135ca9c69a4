"""Generate the golden fixtures in this folder by running the REFERENCE's own
Python code on CPU.

Usage: ``python tests/golden/make_golden.py <path-to-reference-checkout>``

Needs the reference checkout (its ``kernels/w4a16_moe.py`` imports triton,
which only has to be importable).  The reference's ``moe_align_block_size``
asserts ``topk_ids.is_cuda``; a tensor subclass that reports ``is_cuda=True``
lets its pure-torch body run on CPU unchanged.  Outputs:

* ``align_cases.npz``  -- reference moe_align_block_size on seeded ids
* ``config0.npz``      -- configuration-0 inputs, the reference's
  pack_int4_nibbles / dequant_int4_w4a16 / run_reference outputs
* ``routing_known.json`` -- unique-expert counts and weight bytes of the
  reference's make_routing at E=256, top-10, seed 0
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


class _ReportsCuda(torch.Tensor):
    @property
    def is_cuda(self):  # noqa: D401
        return True


ALIGN_CASES = [
    # name, M, topk, E, block_size, seed, kind
    ("cfg0", 4, 2, 8, 16, 0, "uniform"),
    ("m1_e256", 1, 10, 256, 16, 1, "topk"),
    ("m4_e256", 4, 10, 256, 16, 2, "topk"),
    ("m16_e256", 16, 10, 256, 16, 3, "topk"),
    ("m64_e256_bs64", 64, 10, 256, 64, 4, "topk"),
    ("m256_e256_bs128", 256, 10, 256, 128, 5, "topk"),
    ("m1000_e64_bs16", 1000, 6, 64, 16, 6, "topk"),
    ("m3000_e256_bs128", 3000, 10, 256, 128, 7, "topk"),
    ("empty", 0, 10, 256, 16, 8, "topk"),
    ("skew_one_expert", 50, 2, 16, 16, 9, "one"),
    ("dups", 37, 4, 8, 8, 10, "uniform"),
    ("bs1", 20, 3, 12, 1, 11, "uniform"),
    ("int64_ids", 33, 5, 40, 16, 12, "topk64"),
    ("e1000", 200, 8, 1000, 32, 13, "topk"),
]


def _ids_for(M, topk, E, seed, kind):
    g = torch.Generator().manual_seed(seed)
    if kind == "uniform":
        return torch.randint(0, E, (M, topk), generator=g, dtype=torch.int32)
    if kind == "one":
        return torch.full((M, topk), E - 3, dtype=torch.int32)
    logits = torch.randn(M, E, generator=g)
    ids = torch.topk(logits, k=topk, dim=-1).indices
    return ids.to(torch.int64 if kind == "topk64" else torch.int32)


def main(ref: Path) -> None:
    sys.path.insert(0, str(ref))
    from kernels import w4a16_moe as R  # reference kernel module
    from bench import bench_moe as B  # reference bench helpers

    # ---- align ----
    arrays = {}
    for name, M, topk, E, bs, seed, kind in ALIGN_CASES:
        ids = _ids_for(M, topk, E, seed, kind)
        s, e, n = R.moe_align_block_size(ids.as_subclass(_ReportsCuda), bs, E)
        arrays[f"{name}__ids"] = ids.numpy()
        arrays[f"{name}__meta"] = np.array([M, topk, E, bs], dtype=np.int64)
        arrays[f"{name}__sorted"] = torch.Tensor(s).clone().numpy()
        arrays[f"{name}__expert_ids"] = torch.Tensor(e).clone().numpy()
        arrays[f"{name}__num_post"] = torch.Tensor(n).clone().numpy()
    np.savez_compressed(HERE / "align_cases.npz", **arrays)

    # ---- configuration 0 ----
    import importlib.util

    spec = importlib.util.spec_from_file_location(
        "w4a16_b200_synthetic", REPO / "gb10-laguna-s-2.1-w4a16-moe_b200" / "kernels" / "synthetic.py")
    synth = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(synth)
    config0 = synth.config0

    c = config0("cpu")
    w1_packed_ref = B.pack_int4_nibbles(c["w1_codes"])
    w2_packed_ref = B.pack_int4_nibbles(c["w2_codes"])
    w1_deq_bf16 = B.dequant_int4_w4a16(w1_packed_ref, c["w1_s"], 32)
    w2_deq_bf16 = B.dequant_int4_w4a16(w2_packed_ref, c["w2_s"], 32)

    def deq32(packed, s):
        q = B.unpack_int4_nibbles(packed).to(torch.float32) - 8.0
        return q * s.to(torch.float32).repeat_interleave(32, dim=-1)

    E, twoI, H = c["w1_codes"].shape
    I = twoI // 2
    weights32 = B.MoEWeights(
        w1_q=w1_packed_ref, w2_q=w2_packed_ref, w1_scale=c["w1_s"], w2_scale=c["w2_s"],
        w1_ref=deq32(w1_packed_ref, c["w1_s"]), w2_ref=deq32(w2_packed_ref, c["w2_s"]),
        group_size=32, E=E, K=H, N=I,
    )
    out32 = B.run_reference(c["hidden"].to(torch.float32), weights32, c["topk_weights"], c["topk_ids"])
    weights16 = B.MoEWeights(
        w1_q=w1_packed_ref, w2_q=w2_packed_ref, w1_scale=c["w1_s"], w2_scale=c["w2_s"],
        w1_ref=w1_deq_bf16, w2_ref=w2_deq_bf16, group_size=32, E=E, K=H, N=I,
    )
    out16 = B.run_reference(c["hidden"], weights16, c["topk_weights"], c["topk_ids"])
    np.savez_compressed(
        HERE / "config0.npz",
        hidden_bits=c["hidden"].view(torch.int16).numpy().view(np.uint16),
        topk_weights=c["topk_weights"].numpy(),
        topk_ids=c["topk_ids"].numpy(),
        w1_q=c["w1_q"].numpy(), w1_s_bits=c["w1_s"].view(torch.int16).numpy().view(np.uint16),
        w2_q=c["w2_q"].numpy(), w2_s_bits=c["w2_s"].view(torch.int16).numpy().view(np.uint16),
        # The int32 pack-quantized form viewed as uint8 equals the reference's
        # pack_int4_nibbles of the same codes (checked here, recorded as a flag).
        int32_view_equals_nibble_pack=np.array(
            bool(torch.equal(w1_packed_ref, c["w1_q"]) and torch.equal(w2_packed_ref, c["w2_q"]))),
        ref_w1_dequant_bf16_bits_e01=w1_deq_bf16[:2].view(torch.int16).numpy().view(np.uint16),
        ref_w2_dequant_bf16_bits_e01=w2_deq_bf16[:2].view(torch.int16).numpy().view(np.uint16),
        ref_out_fp32=out32.numpy(),
        ref_out_bf16_bits=out16.view(torch.int16).numpy().view(np.uint16),
    )

    # ---- reference make_routing known answers ----
    known = {"E": 256, "topk": 10, "seed": 0, "K": 3072, "N": 1024, "group": 32, "rows": []}
    for M in (1, 4, 16, 64, 256):
        tw, ti = B.make_routing(M, 256, 10, torch.device("cpu"), torch.bfloat16, 0)
        n_act = B.unique_expert_count(ti)
        known["rows"].append({
            "M": M, "unique_experts": n_act,
            "weight_bytes": B.weight_bytes_for_experts(n_act, 3072, 1024, 32),
            "ids_head": ti.reshape(-1)[:20].tolist(),
            "weights_head": [float(v) for v in tw.reshape(-1)[:10]],
        })
    (HERE / "routing_known.json").write_text(json.dumps(known, indent=1) + "\n")
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")), "routing_known.json")


if __name__ == "__main__":
    main(Path(sys.argv[1] if len(sys.argv) > 1 else "/nonexistent"))
