# SPDX-License-Identifier: Apache-2.0
"""W4A16 grouped-MoE for NVIDIA B200 (sm_100a): host side of the C ABI.

Drop-in for the reference module ``kernels/w4a16_moe.py`` (same public names,
argument meanings and return values):

* :func:`repack_weights`  -- reference ``kernels/w4a16_moe.py:63-116``
* :func:`is_repacked`     -- reference ``kernels/w4a16_moe.py:119-121``
* :func:`moe_align_block_size` -- reference ``kernels/w4a16_moe.py:187-290``
* :func:`fused_experts_w4a16`  -- reference ``kernels/w4a16_moe.py:678-909``

All device work happens in ``libw4a16moe_b200.so`` (hand-written sm_100a CUDA,
C ABI in ``include/w4a16_moe_b200.h``), called through ``ctypes`` on the
current torch stream with raw device pointers.  There is no Triton and no CPU
fallback: importing works anywhere, but every compute entry point raises if
the library cannot be loaded or the tensors are not on a CUDA device.

The file is self-contained so that an integration which copies only this
file (``integration/apply.py`` installs it as ``gb10_w4a16_moe.py``) still
works: the library is found through ``W4A16_MOE_B200_LIB`` or next to this
file (``../lib/`` then ``./``).

CUDA-graph capture: after one eager call per shape (which creates the pooled
workspace), every call issues only kernel launches plus one ``torch.empty``
for the returned tensor -- no host sync and no host->device copies.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

# Kept for API compatibility with the reference (kernels/w4a16_moe.py:49-53).
# This library's kernels choose their own tiles; the repacked layout is fixed
# at 16 output rows x 64 k per block.
BLOCK_N: int = 64
BLOCK_K: int = 64
BLOCK_M: int = 16

_GROUP_SIZE_DEFAULT = 32
_ROW_TILE = 16
_CHUNK_K = 64
_CHUNK_BYTES = 512
_CHUNK_SCALES = 32

_LIB_NAME = "libw4a16moe_b200.so"


class W4A16Error(RuntimeError):
    """A C-ABI call returned a nonzero status."""


# ---------------------------------------------------------------------------
# Library loading
# ---------------------------------------------------------------------------

_lib = None
_lib_lock = threading.Lock()


def _candidate_paths() -> list[Path]:
    here = Path(__file__).resolve().parent
    cands = []
    env = os.environ.get("W4A16_MOE_B200_LIB")
    if env:
        cands.append(Path(env))
    cands += [here.parent / "lib" / _LIB_NAME, here / _LIB_NAME, here / "lib" / _LIB_NAME]
    return cands


def library_path() -> Path | None:
    for p in _candidate_paths():
        if p.is_file():
            return p
    return None


def _bind(lib: ctypes.CDLL) -> None:
    c_i64, c_int, c_vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
    lib.w4a16_last_error.restype = ctypes.c_char_p
    lib.w4a16_last_error.argtypes = []
    lib.w4a16_version.restype = c_int
    lib.w4a16_version.argtypes = []
    lib.w4a16_moe_forward_noalloc.restype = c_int
    lib.w4a16_moe_forward_noalloc.argtypes = [
        c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64,
        c_vp, c_vp, c_int, c_i64, c_vp, c_i64, c_vp, c_vp,
    ]
    lib.w4a16_moe_noalloc_max_workspace.restype = c_i64
    lib.w4a16_moe_noalloc_max_workspace.argtypes = []
    lib.w4a16_set_path.restype = c_int
    lib.w4a16_set_path.argtypes = [c_int]
    lib.w4a16_moe_read_status.restype = c_int
    lib.w4a16_moe_read_status.argtypes = [c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, ctypes.POINTER(ctypes.c_int32), c_vp]
    lib.w4a16_set_stage_events.restype = c_int
    lib.w4a16_set_stage_events.argtypes = [ctypes.POINTER(c_vp), c_int]
    lib.w4a16_align_buffer_len.restype = c_i64
    lib.w4a16_align_buffer_len.argtypes = [c_i64, c_i64, c_i64]
    lib.w4a16_moe_align.restype = c_int
    lib.w4a16_moe_align.argtypes = [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp]
    lib.w4a16_moe_align_scratch_bytes.restype = c_i64
    lib.w4a16_moe_align_scratch_bytes.argtypes = [c_i64, c_i64]
    lib.w4a16_moe_align_ex.restype = c_int
    lib.w4a16_moe_align_ex.argtypes = [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp]
    lib.w4a16_repack.restype = c_int
    lib.w4a16_repack.argtypes = [c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp]
    lib.w4a16_topk_softmax.restype = c_int
    lib.w4a16_topk_softmax.argtypes = [c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp]
    lib.w4a16_repack_checkpoint.restype = c_int
    lib.w4a16_repack_checkpoint.argtypes = [c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp]
    lib.w4a16_moe_workspace_size.restype = c_i64
    lib.w4a16_moe_workspace_size.argtypes = [c_i64, c_i64, c_i64, c_i64, c_i64]
    lib.w4a16_moe_forward.restype = c_int
    lib.w4a16_moe_forward.argtypes = [
        c_vp, c_i64, c_i64, c_i64,  # hidden, M, H, ld
        c_vp, c_vp, c_vp, c_vp,  # w13, s13, w2, s2
        c_i64, c_i64,  # E, I
        c_vp, c_vp, c_int, c_i64,  # topk_w, topk_ids, is64, topk
        c_vp, c_i64,  # expert_map, global E
        c_vp, c_vp, c_i64, c_vp,  # out, ws, ws_bytes, stream
    ]


def load_library() -> ctypes.CDLL:
    """Load (once) and return the sm_100a library; raise if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is None:
            path = library_path()
            if path is None:
                raise W4A16Error(
                    f"{_LIB_NAME} not found (looked in "
                    + ", ".join(str(p) for p in _candidate_paths())
                    + "); build it with build.py or set W4A16_MOE_B200_LIB"
                )
            lib = ctypes.CDLL(str(path))
            _bind(lib)
            _lib = lib
    return _lib


def _check(status: int, what: str) -> None:
    if status != 0:
        msg = _lib.w4a16_last_error().decode(errors="replace") if _lib is not None else ""
        raise W4A16Error(f"{what} failed (status {status}): {msg}")


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise AssertionError("all tensors must live on a CUDA device (no CPU fallback)")


# ---------------------------------------------------------------------------
# Repack (load time)
# ---------------------------------------------------------------------------


def repack_weights(
    w_q: torch.Tensor,
    scales: torch.Tensor,
    block_n: int = BLOCK_N,
) -> tuple[torch.Tensor, torch.Tensor]:
    """One-time transform of vLLM-layout int4 weights into this library's layout.

    Parameters
    ----------
    w_q:
        ``(E, N_out, K_in//2)`` uint8, low nibble = even K, high nibble = odd K,
        stored value = q + 8 (reference ``kernels/w4a16_moe.py:63-87``).
    scales:
        ``(E, N_out, K_in//group_size)`` bf16 group scales; group_size must be
        a multiple of 32 (larger groups are stored replicated, exactly).
    block_n:
        Accepted for signature compatibility; the layout is fixed.

    Returns
    -------
    w_rep : ``(E, N_out//16, K_in//64, 512)`` uint8 (fragment-major)
    s_rep : ``(E, N_out//16, K_in//64, 32)`` bf16
    """
    del block_n
    assert w_q.ndim == 3 and scales.ndim == 3
    _require_cuda(w_q, scales)
    E, N_out, K_half = w_q.shape
    assert scales.shape[0] == E and scales.shape[1] == N_out
    assert w_q.dtype == torch.uint8, "packed weights must be uint8"
    assert scales.dtype == torch.bfloat16, "scales must be bf16"
    K = 2 * K_half
    num_groups = scales.shape[2]
    assert num_groups > 0 and K % num_groups == 0
    group = K // num_groups
    lib = load_library()
    w_q = w_q.contiguous()
    scales = scales.contiguous()
    w_rep = torch.empty((E, N_out // _ROW_TILE, K // _CHUNK_K, _CHUNK_BYTES), dtype=torch.uint8, device=w_q.device)
    s_rep = torch.empty((E, N_out // _ROW_TILE, K // _CHUNK_K, _CHUNK_SCALES), dtype=torch.bfloat16, device=w_q.device)
    with torch.cuda.device(w_q.device):
        _check(
            lib.w4a16_repack(
                w_q.data_ptr(), scales.data_ptr(), E, N_out, K, group,
                w_rep.data_ptr(), s_rep.data_ptr(), _stream_ptr(w_q.device),
            ),
            "w4a16_repack",
        )
    return w_rep, s_rep


def repack_checkpoint(w_packed: torch.Tensor, scales: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Library layout straight from vLLM's ``create_weights`` tensors.

    ``w_packed``: ``(E, K_in//8, N_out)`` int32 compressed-tensors
    ``pack-quantized`` codes (is_transposed=True: 8 codes of one output row
    per int32 along K, code j at bits 4j); ``scales``: ``(E, K_in//group,
    N_out)`` bf16.  Equals ``repack_weights(w_packed.transpose(1, 2)
    .contiguous().view(torch.uint8), scales.transpose(1, 2).contiguous())``
    (the reference's load path, ``integration/apply.py:100-105``) without the
    transposed copies.
    """
    assert w_packed.ndim == 3 and scales.ndim == 3
    _require_cuda(w_packed, scales)
    assert w_packed.dtype == torch.int32, "packed weights must be int32"
    assert scales.dtype == torch.bfloat16, "scales must be bf16"
    E, K8, N_out = w_packed.shape
    K = 8 * K8
    assert scales.shape[0] == E and scales.shape[2] == N_out
    num_groups = scales.shape[1]
    assert num_groups > 0 and K % num_groups == 0
    group = K // num_groups
    w_packed = w_packed.contiguous()
    scales = scales.contiguous()
    dev = w_packed.device
    w_rep = torch.empty((E, N_out // _ROW_TILE, K // _CHUNK_K, _CHUNK_BYTES), dtype=torch.uint8, device=dev)
    s_rep = torch.empty((E, N_out // _ROW_TILE, K // _CHUNK_K, _CHUNK_SCALES), dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        _check(
            load_library().w4a16_repack_checkpoint(
                w_packed.data_ptr(), scales.data_ptr(), E, N_out, K, group,
                w_rep.data_ptr(), s_rep.data_ptr(), _stream_ptr(dev),
            ),
            "w4a16_repack_checkpoint",
        )
    return w_rep, s_rep


def topk_softmax(logits: torch.Tensor, topk: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Router on the GPU: ``(topk_weights [M, topk] fp32, topk_ids [M, topk]
    int32)`` = softmax over the top-k of fp32 ``logits [M, E]``, ids in
    descending logit order -- the reference benchmark's routing
    (``bench/bench_moe.py:225-231``)."""
    _require_cuda(logits)
    assert logits.ndim == 2 and logits.dtype == torch.float32, "logits must be fp32 [M, E]"
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    M, E = logits.shape
    dev = logits.device
    w = torch.empty((M, topk), dtype=torch.float32, device=dev)
    ids = torch.empty((M, topk), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _check(load_library().w4a16_topk_softmax(logits.data_ptr(), M, E, logits.stride(0), topk, w.data_ptr(),
                                                 ids.data_ptr(), _stream_ptr(dev)), "w4a16_topk_softmax")
    return w, ids


def is_repacked(w_q: torch.Tensor) -> bool:
    """True if ``w_q`` is in the 4-D layout from :func:`repack_weights`."""
    return w_q.ndim == 4


# ---------------------------------------------------------------------------
# Routing
# ---------------------------------------------------------------------------

# (device, n_tok, num_experts, block_size) -> output buffers, reused per call
# exactly like the reference's _ALIGN_CACHE (kernels/w4a16_moe.py:135).
_ALIGN_CACHE: dict[tuple, tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = {}


def moe_align_block_size(
    topk_ids: torch.Tensor,
    block_size: int,
    num_experts: int,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Sort token slots by expert and pad each expert to ``block_size``.

    Bit-exact with the reference (``kernels/w4a16_moe.py:187-290``); one GPU
    kernel instead of ~12 torch ops.  As in the reference the returned tensors
    are pooled per shape and overwritten by the next call of the same shape.

    Returns
    -------
    sorted_token_ids : int32 ``[max_num_tokens_padded]`` (padding = M*topk)
    expert_ids : int32 ``[max_num_m_blocks]`` (-1 for unused trailing blocks)
    num_tokens_post_padded : int32 ``[1]``
    """
    assert topk_ids.is_cuda, "topk_ids must be on CUDA for graph capture"
    assert topk_ids.ndim == 2
    M, topk = topk_ids.shape
    n_tok = M * topk
    lib = load_library()
    device = topk_ids.device
    key = (str(device), n_tok, num_experts, block_size)
    bufs = _ALIGN_CACHE.get(key)
    if bufs is None:
        P = int(lib.w4a16_align_buffer_len(n_tok, num_experts, block_size))
        assert P >= 0, "bad align sizes"
        with torch.cuda.device(device):
            sb = int(lib.w4a16_moe_align_scratch_bytes(n_tok, num_experts))
        bufs = (
            torch.empty(P, dtype=torch.int32, device=device),
            torch.empty(P // block_size, dtype=torch.int32, device=device),
            torch.empty(1, dtype=torch.int32, device=device),
            # multi-CTA scratch (zero-filled once, left clean by every call)
            torch.zeros(max(sb, 0) + 256, dtype=torch.uint8, device=device) if sb > 0 else None,
        )
        _ALIGN_CACHE[key] = bufs
    ids = topk_ids
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.to(torch.int32)
    ids = ids.contiguous()
    with torch.cuda.device(device):
        _check(
            lib.w4a16_moe_align_ex(
                ids.data_ptr(), 1 if ids.dtype == torch.int64 else 0, M, topk, num_experts,
                block_size, bufs[0].data_ptr(), bufs[1].data_ptr(), bufs[2].data_ptr(),
                _ws_ptr(bufs[3]) if bufs[3] is not None else None,
                bufs[3].numel() - 256 if bufs[3] is not None else 0,
                _stream_ptr(device),
            ),
            "w4a16_moe_align",
        )
    return bufs[:3]


# ---------------------------------------------------------------------------
# Fused experts
# ---------------------------------------------------------------------------

# (device, M, topk, E, H, I) -> zero-initialised uint8 workspace (the forward
# keeps its self-cleaning counters at zero between calls).
_WS_CACHE: dict[tuple, torch.Tensor] = {}


def _device_key(device: torch.device | str) -> str:
    """Cache key of a device: "cuda" and "cuda:<current>" name the same one."""
    d = torch.device(device)
    if d.type == "cuda" and d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    return str(d)


def _workspace(device: torch.device, M: int, topk: int, E: int, H: int, I: int) -> torch.Tensor:
    key = (_device_key(device), M, topk, E, H, I)
    ws = _WS_CACHE.get(key)
    if ws is None:
        nbytes = int(load_library().w4a16_moe_workspace_size(M, topk, E, H, I))
        assert nbytes > 0, "bad workspace sizes"
        ws = torch.zeros(nbytes + 256, dtype=torch.uint8, device=device)
        _WS_CACHE[key] = ws
    return ws


def _ws_ptr(ws: torch.Tensor) -> int:
    p = ws.data_ptr()
    return (p + 255) // 256 * 256


def set_stage_events(events: list | None) -> None:
    """Profiling hook: record ``events`` (torch.cuda.Event, enable_timing) at the
    forward's stage boundaries -- before routing, after routing, after w13,
    after w2 -- on the calling thread.  ``None`` disables it."""
    lib = load_library()
    if not events:
        _check(lib.w4a16_set_stage_events(None, 0), "w4a16_set_stage_events")
        return
    for ev in events:
        ev.record()  # materialise the underlying cudaEvent_t
    arr = (ctypes.c_void_p * len(events))(*[ev.cuda_event for ev in events])
    _check(lib.w4a16_set_stage_events(arr, len(events)), "w4a16_set_stage_events")


def set_path(path: str) -> None:
    """Select the forward implementation for the calling thread: ``"auto"``
    (fused persistent decode kernel for small M, tensor-core kernels
    otherwise), ``"general"`` (multi-kernel CUDA-core path) or ``"prefill"``
    (the tensor-core path at any M)."""
    codes = {"auto": 0, "general": 1, "prefill": 2}
    _check(load_library().w4a16_set_path(codes[path]), "w4a16_set_path")


def read_status(hidden_shape: tuple[int, int], topk: int, num_experts: int, intermediate: int,
                device: torch.device | str = "cuda") -> int:
    """Read and clear the error bits recorded in the pooled workspace of a
    forward shape (0 = no bounded wait timed out).  Synchronises."""
    M, H = hidden_shape
    ws = _WS_CACHE.get((_device_key(device), M, topk, num_experts, H, intermediate))
    if ws is None:
        return 0
    out = ctypes.c_int32(0)
    _check(load_library().w4a16_moe_read_status(_ws_ptr(ws), M, topk, num_experts, H, intermediate,
                                                ctypes.byref(out), _stream_ptr(ws.device)),
           "w4a16_moe_read_status")
    return int(out.value)


def clear_workspace_cache() -> None:
    """Drop pooled workspaces and align buffers (e.g. before empty_cache())."""
    _WS_CACHE.clear()
    _ALIGN_CACHE.clear()


def fused_experts_w4a16(
    hidden: torch.Tensor,
    w1_q: torch.Tensor,
    w2_q: torch.Tensor,
    w1_scale: torch.Tensor,
    w2_scale: torch.Tensor,
    topk_weights: torch.Tensor,
    topk_ids: torch.Tensor,
    group_size: int = _GROUP_SIZE_DEFAULT,
    *,
    block_m: int = BLOCK_M,
    block_n: int = BLOCK_N,
    block_k: int = BLOCK_K,
    expert_map: torch.Tensor | None = None,
    global_num_experts: int = -1,
    activation: str = "silu",
    apply_router_weight_on_input: bool = False,
    inplace: bool = False,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Fused W4A16 grouped-MoE experts (w13 + SiLU-mul + w2 + weighted top-k sum).

    Same call surface as the reference (``kernels/w4a16_moe.py:678-691``).

    Parameters
    ----------
    hidden:
        ``[M, K]`` bf16 activations (row stride may exceed K).
    w1_q, w1_scale:
        Either vLLM layout ``(E, 2N, K//2)`` / ``(E, 2N, K//group)`` or the 4-D
        layout from :func:`repack_weights`.  Prefer repacked (done once).
    w2_q, w2_scale:
        ``(E, K, N//2)`` / ``(E, K, N//group)`` or repacked 4-D.
    topk_weights:
        ``[M, topk]`` routing weights (fp32; other float types are cast).
    topk_ids:
        ``[M, topk]`` int32 (or int64) expert indices.
    group_size:
        Group size of 3-D scales (inferred from their shape; checked).
    expert_map, global_num_experts:
        Optional vLLM expert-parallel table (global id -> local id or -1).
        Slots mapped to -1 contribute nothing; tokens with no local slot
        return zero rows.  (Extension: the reference drops these arguments.)
    block_m, block_n, block_k:
        Accepted for compatibility; tiles are chosen by the library.
    out:
        Optional preallocated ``[M, K]`` bf16 output.

    Returns
    -------
    Tensor
        ``[M, K]`` bf16, a fresh tensor unless ``out``/``inplace`` is given.
    """
    del block_m, block_n, block_k
    assert hidden.ndim == 2
    _require_cuda(hidden, topk_ids, topk_weights)
    assert topk_ids.shape == topk_weights.shape
    assert hidden.dtype == torch.bfloat16, "bf16 activations required"
    if activation != "silu":
        raise NotImplementedError(f"activation {activation!r} is not supported (silu only)")
    M, K = hidden.shape
    topk = int(topk_ids.shape[1]) if topk_ids.ndim == 2 else 1
    device = hidden.device

    if not is_repacked(w1_q):
        assert w1_scale.ndim == 3 and 2 * w1_q.shape[2] == K
        assert w1_scale.shape[2] * group_size == K, "w1_scale groups do not match group_size"
        w1_q, w1_scale = repack_weights(w1_q, w1_scale)
    if not is_repacked(w2_q):
        assert w2_scale.ndim == 3 and w2_scale.shape[2] * group_size == 2 * w2_q.shape[2], (
            "w2_scale groups do not match group_size"
        )
        w2_q, w2_scale = repack_weights(w2_q, w2_scale)

    assert w1_q.dtype == torch.uint8 and w1_q.shape[-1] == _CHUNK_BYTES, (
        "w1_q is 4-D but not in this library's repacked layout"
    )
    assert w2_q.dtype == torch.uint8 and w2_q.shape[-1] == _CHUNK_BYTES, (
        "w2_q is 4-D but not in this library's repacked layout"
    )
    E, n_rt13, n_ch13, _ = w1_q.shape
    assert n_ch13 * _CHUNK_K == K, f"K mismatch: packed {n_ch13 * _CHUNK_K} vs hidden {K}"
    twoN = n_rt13 * _ROW_TILE
    N = twoN // 2
    E2, n_rt2, n_ch2, _ = w2_q.shape
    assert E2 == E and n_ch2 * _CHUNK_K == N and n_rt2 * _ROW_TILE == K
    assert w1_scale.shape == (E, n_rt13, n_ch13, _CHUNK_SCALES)
    assert w2_scale.shape == (E, n_rt2, n_ch2, _CHUNK_SCALES)
    _require_cuda(w1_q, w2_q, w1_scale, w2_scale)

    if apply_router_weight_on_input:
        # vLLM semantics (topk == 1): scale the input rows, unit router weight.
        assert topk == 1, "apply_router_weight_on_input requires topk == 1"
        hidden = (hidden.float() * topk_weights.reshape(M, 1).float()).to(torch.bfloat16)
        topk_weights = torch.ones_like(topk_weights, dtype=torch.float32)

    tw = topk_weights
    if tw.dtype != torch.float32:
        tw = tw.to(torch.float32)
    tw = tw.contiguous()
    ids = topk_ids
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.to(torch.int32)
    ids = ids.contiguous()
    if hidden.stride(1) != 1:
        hidden = hidden.contiguous()
    emap_ptr, gE = 0, -1
    if expert_map is not None:
        _require_cuda(expert_map)
        emap = expert_map if expert_map.dtype == torch.int32 else expert_map.to(torch.int32)
        emap = emap.contiguous()
        emap_ptr = emap.data_ptr()
        gE = int(global_num_experts) if global_num_experts > 0 else int(emap.numel())

    if out is None:
        out = torch.empty((M, K), dtype=torch.bfloat16, device=device)
    else:
        assert out.shape == (M, K) and out.dtype == torch.bfloat16 and out.is_contiguous()
    if M == 0:
        return out
    lib = load_library()
    ws = _workspace(device, M, topk, E, K, N)
    with torch.cuda.device(device):
        _check(
            lib.w4a16_moe_forward(
                hidden.data_ptr(), M, K, hidden.stride(0),
                w1_q.data_ptr(), w1_scale.data_ptr(), w2_q.data_ptr(), w2_scale.data_ptr(),
                E, N, tw.data_ptr(), ids.data_ptr(), 1 if ids.dtype == torch.int64 else 0, topk,
                emap_ptr, gE, out.data_ptr(), _ws_ptr(ws), ws.numel() - 256, _stream_ptr(device),
            ),
            "w4a16_moe_forward",
        )
    if inplace:
        hidden.copy_(out)
        return hidden
    return out
