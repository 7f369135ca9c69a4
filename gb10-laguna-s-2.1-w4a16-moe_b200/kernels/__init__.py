# W4A16 grouped-MoE kernels for B200 (sm_100a).
# Mirrors the reference package's lazy re-export (kernels/__init__.py:3-11).
__all__ = [
    "fused_experts_w4a16",
    "repack_weights",
    "moe_align_block_size",
    "is_repacked",
    "repack_checkpoint",
    "topk_softmax",
]


def __getattr__(name: str):
    if name in __all__:
        from kernels import w4a16_moe

        return getattr(w4a16_moe, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
