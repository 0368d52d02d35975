"""FP16 paged-KV GQA decode attention on B200 (the hot path).

Drop-in for ``paged_decode_attention_triton`` (reference: src/bpt/triton_fp16.py:183-247):
same arguments, same ``num_splits`` meaning (None = heuristic, 1 = single pass, n = n-way
split), same layout, fresh output tensor, launch on the current torch stream. Behind it is the
C ABI ``bpt_decode_fp16`` (include/bpt.h), hand-written sm_100a CUDA.

Differences from the reference launcher, all deliberate:
  * no ``int(seq_lens.min())`` device->host sync (triton_fp16.py:201): a sequence of length 0
    is allowed and yields zeros (what the reference oracle returns for it), so the call can
    be captured in a CUDA graph;
  * the scratch for split partials is one workspace tensor (or the caller's ``workspace``);
  * the heuristic split count is tuned for B200 (``bpt_plan_splits``).
"""
import functools
import math
import os
from typing import Optional

import torch

from . import _lib
from ._lib import BptArgumentError, BptError, BptUnsupportedError

CHECKS = os.environ.get("BPT_CHECKS", "0") not in ("", "0")

DEVICE_FLAGS = {1: "block_table entry outside [0, num_blocks)",
                2: "seq_len > max_blocks * block_size",
                4: "pipeline wait timed out",
                8: "negative seq_len"}


@functools.lru_cache(maxsize=None)
def _sm_count(device_index: int) -> int:
    """SM count of a device (reference: src/bpt/triton_fp16.py:170-172)."""
    return torch.cuda.get_device_properties(device_index).multi_processor_count


def _require(cond: bool, msg: str):
    if not cond:
        raise BptArgumentError(msg)


def _pow2(x: int) -> bool:
    return x > 0 and (x & (x - 1)) == 0


def choose_num_splits(batch: int, kv_heads: int, block_size: int, max_pages: int,
                      sm_count: int) -> int:
    """Heuristic split count (reference: src/bpt/triton_fp16.py:175-180), B200-tuned."""
    return int(_lib.lib().bpt_plan_splits(batch, kv_heads, block_size, max_pages, sm_count))


def effective_splits(batch: int, kv_heads: int, block_size: int, max_pages: int,
                     num_splits: Optional[int], sm_count: int) -> int:
    return int(_lib.lib().bpt_effective_splits(batch, kv_heads, block_size, max_pages,
                                               int(num_splits or 0), sm_count))


def workspace_bytes(batch: int, q_heads: int, head_dim: int, splits: int) -> int:
    return int(_lib.lib().bpt_decode_workspace_bytes(batch, q_heads, head_dim, splits))


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def check_device_flags(workspace: torch.Tensor, what: str = "decode"):
    """Read the device-check word at the start of a workspace (synchronises)."""
    flags = int(workspace[:4].view(torch.int32).item())
    if flags:
        names = [v for k, v in DEVICE_FLAGS.items() if flags & k]
        raise BptError(-8, f"{what}: device check failed: " + "; ".join(names))


def _validate_common(q, k_cache, v_cache, block_table, seq_lens):
    _require(q.dim() == 3, "q must be [B, Hq, D]")
    _require(k_cache.dim() == 4 and v_cache.dim() == 4,
             "k_cache/v_cache must be [num_blocks, block_size, Hkv, D]")
    _require(k_cache.shape == v_cache.shape, "k_cache and v_cache shapes differ")
    B, Hq, D = q.shape
    _, block_size, Hkv, Dk = k_cache.shape
    _require(Dk == D, "head_dim of q and cache differ")
    _require(Hq % Hkv == 0, "q heads must be a multiple of kv heads")
    _require(block_table.dim() == 2 and block_table.shape[0] == B, "block_table must be [B, *]")
    _require(seq_lens.dim() == 1 and seq_lens.shape[0] == B, "seq_lens must be [B]")
    _require(block_table.dtype == torch.int32 and seq_lens.dtype == torch.int32,
             "block_table and seq_lens must be int32")
    dev = q.device
    _require(dev.type == "cuda", "bpt runs on CUDA tensors only (no CPU fallback)")
    for t, n in ((k_cache, "k_cache"), (v_cache, "v_cache"), (block_table, "block_table"),
                 (seq_lens, "seq_lens")):
        _require(t.device == dev, f"{n} is on {t.device}, q on {dev}")
    _require(block_table.stride(1) == 1 or block_table.shape[1] <= 1,
             "block_table rows must be contiguous")
    _require(seq_lens.is_contiguous(), "seq_lens must be contiguous")
    return B, Hq, D, block_size, Hkv


def paged_decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           block_table: torch.Tensor, seq_lens: torch.Tensor,
                           scale: Optional[float] = None, num_splits: Optional[int] = None,
                           *, out: Optional[torch.Tensor] = None,
                           workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """GQA decode over an FP16 paged KV cache -> [B, Hq, D] fp16.

    q [B, Hq, D]; k_cache/v_cache [num_blocks, block_size, Hkv, D]; block_table
    [B, max_blocks] int32; seq_lens [B] int32 (0 allowed). Preconditions follow
    src/bpt/triton_fp16.py:195-200 and raise ``BptArgumentError`` (an AssertionError).
    """
    B, Hq, D, block_size, Hkv = _validate_common(q, k_cache, v_cache, block_table, seq_lens)
    _require(q.dtype == k_cache.dtype == v_cache.dtype == torch.float16,
             "q, k_cache and v_cache must be float16")
    _require(_pow2(D) and D >= 16, "head_dim must be a power of two >= 16")
    _require(_pow2(block_size) and block_size >= 16, "block_size must be a power of two >= 16")
    _require(q.stride(2) == 1 and k_cache.stride(3) == 1 and v_cache.stride(3) == 1,
             "innermost (head_dim) stride must be 1")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    dev = q.device
    max_blocks = block_table.shape[1]
    S = effective_splits(B, Hkv, block_size, max_blocks, num_splits, _sm_count(dev.index or 0))
    need = workspace_bytes(B, Hq, D, S)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    if CHECKS:
        workspace[:4].zero_()
    if out is None:
        out = torch.empty_like(q)
    _require(out.shape == q.shape and out.dtype == torch.float16 and out.stride(2) == 1,
             "out must be a float16 [B, Hq, D] tensor with unit inner stride")
    rc = _lib.lib().bpt_decode_fp16(
        q.data_ptr(), q.stride(0), q.stride(1),
        k_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
        v_cache.data_ptr(), v_cache.stride(0), v_cache.stride(1), v_cache.stride(2),
        k_cache.shape[0],
        block_table.data_ptr(), block_table.stride(0),
        seq_lens.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1),
        B, Hq, Hkv, D, block_size, max_blocks,
        float(scale), int(num_splits or 0), _sm_count(dev.index or 0),
        workspace.data_ptr(), workspace.numel() * workspace.element_size(),
        _stream_handle(dev))
    _lib.check(rc, "bpt_decode_fp16")
    if CHECKS:
        check_device_flags(workspace, "bpt_decode_fp16")
    return out


def paged_decode_attention_partial(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                                   block_table: torch.Tensor, seq_lens: torch.Tensor,
                                   scale: Optional[float] = None, num_splits: Optional[int] = None,
                                   *, o_part: Optional[torch.Tensor] = None,
                                   lse: Optional[torch.Tensor] = None,
                                   status: Optional[torch.Tensor] = None):
    """Stage 1 only: per-split normalised partial outputs and their log2-sum-exp.

    Returns (o_part [B, Hq, S, D] fp32, lse [B, Hq, S] fp32 in log2 units). The split kernel of
    src/bpt/triton_fp16.py:83-144 (which writes natural-log lse); a sequence-sharded caller
    merges these with ``merge_partials`` / ``merge_states`` after exchanging them.
    """
    B, Hq, D, block_size, Hkv = _validate_common(q, k_cache, v_cache, block_table, seq_lens)
    _require(q.dtype == k_cache.dtype == v_cache.dtype == torch.float16,
             "q, k_cache and v_cache must be float16")
    _require(q.stride(2) == 1 and k_cache.stride(3) == 1 and v_cache.stride(3) == 1,
             "innermost (head_dim) stride must be 1")
    dev = q.device
    max_blocks = block_table.shape[1]
    S = effective_splits(B, Hkv, block_size, max_blocks, num_splits, _sm_count(dev.index or 0))
    if o_part is None:
        o_part = torch.empty(B, Hq, S, D, dtype=torch.float32, device=dev)
    if lse is None:
        lse = torch.empty(B, Hq, S, dtype=torch.float32, device=dev)
    _require(o_part.shape == (B, Hq, S, D) and o_part.is_contiguous()
             and o_part.dtype == torch.float32, f"o_part must be contiguous fp32 {(B, Hq, S, D)}")
    _require(lse.shape == (B, Hq, S) and lse.is_contiguous() and lse.dtype == torch.float32,
             f"lse must be contiguous fp32 {(B, Hq, S)}")
    rc = _lib.lib().bpt_decode_fp16_partial(
        q.data_ptr(), q.stride(0), q.stride(1),
        k_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
        v_cache.data_ptr(), v_cache.stride(0), v_cache.stride(1), v_cache.stride(2),
        k_cache.shape[0], block_table.data_ptr(), block_table.stride(0), seq_lens.data_ptr(),
        B, Hq, Hkv, D, block_size, max_blocks,
        float(scale if scale is not None else 1.0 / math.sqrt(D)), S,
        o_part.data_ptr(), lse.data_ptr(), status.data_ptr() if status is not None else None,
        _stream_handle(dev))
    _lib.check(rc, "bpt_decode_fp16_partial")
    return o_part, lse


def merge_partials(o_part: torch.Tensor, lse: torch.Tensor,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Stage 2: LSE-weighted merge of [B, Hq, S, D] partials -> fp16 [B, Hq, D]
    (src/bpt/triton_fp16.py:147-163)."""
    B, Hq, S, D = o_part.shape
    _require(o_part.is_contiguous() and lse.is_contiguous() and lse.shape == (B, Hq, S),
             "o_part [B, Hq, S, D] and lse [B, Hq, S] must be contiguous")
    if out is None:
        out = torch.empty(B, Hq, D, dtype=torch.float16, device=o_part.device)
    rc = _lib.lib().bpt_merge_partials(o_part.data_ptr(), lse.data_ptr(), B, Hq, D, S,
                                       out.data_ptr(), out.stride(0), out.stride(1),
                                       _stream_handle(o_part.device))
    _lib.check(rc, "bpt_merge_partials")
    return out


def merge_states(o_part: torch.Tensor, lse: torch.Tensor):
    """Merge [B, Hq, S, D] partials into one fp32 state per (b, q head): (o [B, Hq, D],
    lse [B, Hq]) in log2 units."""
    B, Hq, S, D = o_part.shape
    _require(o_part.is_contiguous() and lse.is_contiguous() and lse.shape == (B, Hq, S),
             "o_part [B, Hq, S, D] and lse [B, Hq, S] must be contiguous")
    o = torch.empty(B, Hq, D, dtype=torch.float32, device=o_part.device)
    l2 = torch.empty(B, Hq, dtype=torch.float32, device=o_part.device)
    return merge_states_into(o_part, lse, o, l2)


def merge_states_into(o_part: torch.Tensor, lse: torch.Tensor, o: torch.Tensor,
                      l2: torch.Tensor):
    """``merge_states`` writing into caller tensors (contiguous fp32 [B, Hq, D], [B, Hq])."""
    B, Hq, S, D = o_part.shape
    _require(o_part.is_contiguous() and lse.is_contiguous() and lse.shape == (B, Hq, S),
             "o_part [B, Hq, S, D] and lse [B, Hq, S] must be contiguous")
    _require(o.shape == (B, Hq, D) and o.is_contiguous() and o.dtype == torch.float32 and
             l2.shape == (B, Hq) and l2.is_contiguous() and l2.dtype == torch.float32,
             "o must be contiguous fp32 [B, Hq, D] and l2 fp32 [B, Hq]")
    rc = _lib.lib().bpt_merge_states(o_part.data_ptr(), lse.data_ptr(), B, Hq, D, S,
                                     o.data_ptr(), l2.data_ptr(), _stream_handle(o_part.device))
    _lib.check(rc, "bpt_merge_states")
    return o, l2


__all__ = ["paged_decode_attention", "paged_decode_attention_partial", "merge_partials",
           "merge_states", "choose_num_splits", "effective_splits", "workspace_bytes",
           "BptError", "BptArgumentError", "BptUnsupportedError", "check_device_flags"]
