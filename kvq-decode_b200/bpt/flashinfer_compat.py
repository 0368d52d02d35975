"""FlashInfer-compatible batch decode over bpt's kernels (a drop-in for serving engines that
call FlashInfer's paged decode, e.g. vLLM's FlashInfer attention backend).

No counterpart in the reference (its README plans a vLLM/FlashInfer-compatible backend as a
later milestone). ``BatchDecodeWithPagedKVCacheWrapper`` keeps FlashInfer's plan/run split and
argument meaning:

* ``plan(indptr, indices, last_page_len, num_qo_heads, num_kv_heads, head_dim, page_size, ...)``
  takes the CSR page lists (sequence b owns pages ``indices[indptr[b]:indptr[b+1]]``, the last
  one holding ``last_page_len[b]`` tokens). It turns them into bpt's block table
  [B, max_pages] int32 and seq_lens [B] int32 on the device, and fixes the split count. Like
  FlashInfer's plan it is a host-side step: it reads indptr on the host.
* ``run(q, paged_kv_cache, out=None, lse=None, return_lse=False)`` decodes one token per
  sequence. The cache is either one tensor ``[P, 2, page_size, Hkv, D]`` (layout "NHD") or
  ``[P, 2, Hkv, page_size, D]`` ("HND"), or a (k, v) tuple of ``[P, page_size, Hkv, D]`` /
  ``[P, Hkv, page_size, D]``. All of these are strided views that bpt's tensor maps read in
  place. ``return_lse`` returns the log-sum-exp of the scaled logits in base 2.

Supported: fp16 q / cache, head_dim 16-256, any group of at most 8 q heads per kv head, page
sizes that are powers of two from 16 to 256. Rejected with ``BptArgumentError``: position
encodings applied inside attention (ROPE_LLAMA / ALIBI), sliding windows, logit soft-capping,
fp8 caches. bpt's KIVI formats have their own API (``bpt.quant``).
"""
from typing import Optional, Tuple, Union

import torch

from ._lib import BptArgumentError
from .decode import (_require, _sm_count, effective_splits, merge_states_into,
                     paged_decode_attention, paged_decode_attention_partial, workspace_bytes)


def csr_to_block_table(indptr: torch.Tensor, indices: torch.Tensor, last_page_len: torch.Tensor,
                       page_size: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
    """FlashInfer's CSR page lists -> (block_table [B, max_pages] int32, seq_lens [B] int32) on
    `device`. Sequence b owns pages indices[indptr[b]:indptr[b+1]] in order; its last page
    holds last_page_len[b] tokens; a sequence without pages has length 0. Unused table slots are
    0 (never read). indptr is read on the host."""
    ip = indptr.to("cpu", torch.int64)
    B = ip.numel() - 1
    _require(B >= 0, "indptr must hold batch_size + 1 entries")
    pages = ip[1:] - ip[:-1]
    _require(bool((pages >= 0).all()), "indptr must be non-decreasing")
    max_pages = max(int(pages.max()) if B > 0 else 0, 1)
    ind = indices.to(device, torch.int32)
    ipd = ip.to(device)
    pg = pages.to(device)
    col = torch.arange(max_pages, device=device, dtype=torch.int64)
    pos = (ipd[:-1, None] + col[None, :]).clamp(max=max(ind.numel() - 1, 0))
    has = col[None, :] < pg[:, None]
    if ind.numel():
        table = torch.where(has, ind[pos], torch.zeros((), dtype=torch.int32, device=device))
    else:
        table = torch.zeros(B, max_pages, dtype=torch.int32, device=device)
    lpl = last_page_len.to(device, torch.int64)
    seq = torch.where(pg > 0, (pg - 1) * page_size + lpl, torch.zeros_like(pg))
    return table.to(torch.int32).contiguous(), seq.to(torch.int32).contiguous()


class BatchDecodeWithPagedKVCacheWrapper:
    def __init__(self, float_workspace_buffer: torch.Tensor, kv_layout: str = "NHD",
                 use_cuda_graph: bool = False, use_tensor_cores: bool = False, **_ignored):
        _require(kv_layout in ("NHD", "HND"), f"unsupported kv_layout {kv_layout!r}")
        self._ws = float_workspace_buffer
        self._layout = kv_layout
        self._planned = False

    # ------------------------------------------------------------------------ plan
    def plan(self, indptr: torch.Tensor, indices: torch.Tensor, last_page_len: torch.Tensor,
             num_qo_heads: int, num_kv_heads: int, head_dim: int, page_size: int,
             pos_encoding_mode: str = "NONE", window_left: int = -1,
             logits_soft_cap: Optional[float] = None,
             q_data_type: Union[str, torch.dtype] = "float16",
             kv_data_type: Union[str, torch.dtype, None] = None,
             sm_scale: Optional[float] = None, **_ignored) -> None:
        _require(pos_encoding_mode == "NONE",
                 "position encodings inside attention are not supported (apply RoPE to q/k)")
        _require(window_left in (-1, None), "sliding-window decode is not supported")
        _require(not logits_soft_cap, "logit soft-capping is not supported")
        for name, dt in (("q_data_type", q_data_type), ("kv_data_type", kv_data_type)):
            _require(dt in (None, "float16", torch.float16), f"{name} must be float16")
        _require(num_qo_heads % num_kv_heads == 0, "num_qo_heads % num_kv_heads != 0")
        dev = indices.device if indices.is_cuda else torch.device("cuda",
                                                                   torch.cuda.current_device())
        self._bt, self._sl = csr_to_block_table(indptr, indices, last_page_len, page_size, dev)
        B, max_pages = self._bt.shape
        self._B, self._Hq, self._Hkv, self._D = B, num_qo_heads, num_kv_heads, head_dim
        self._page = page_size
        self._scale = sm_scale
        self._S = effective_splits(B, num_kv_heads, page_size, max_pages, None,
                                   _sm_count(dev.index or 0))
        need = workspace_bytes(B, num_qo_heads, head_dim, self._S)
        ws = self._ws
        if ws is not None and ws.is_cuda and ws.numel() * ws.element_size() >= need:
            self._ws_view = ws.view(torch.uint8).reshape(-1)[:need]
        else:
            self._ws_view = torch.empty(need, dtype=torch.uint8, device=dev)
        self._planned = True

    # ------------------------------------------------------------------------ run
    def _kv(self, paged_kv_cache) -> Tuple[torch.Tensor, torch.Tensor]:
        if isinstance(paged_kv_cache, (tuple, list)):
            k, v = paged_kv_cache
        else:
            _require(paged_kv_cache.dim() == 5 and paged_kv_cache.shape[1] == 2,
                     "paged_kv_cache must be [num_pages, 2, ...] or a (k, v) tuple")
            k, v = paged_kv_cache[:, 0], paged_kv_cache[:, 1]
        if self._layout == "HND":   # [P, Hkv, page, D] -> strided [P, page, Hkv, D] view
            k, v = k.transpose(1, 2), v.transpose(1, 2)
        _require(tuple(k.shape[1:]) == (self._page, self._Hkv, self._D),
                 f"cache pages must be {(self._page, self._Hkv, self._D)} in layout "
                 f"{self._layout}, got {tuple(k.shape[1:])}")
        return k, v

    def run(self, q: torch.Tensor, paged_kv_cache, *args, out: Optional[torch.Tensor] = None,
            lse: Optional[torch.Tensor] = None, return_lse: bool = False, **_ignored):
        _require(self._planned, "plan() must be called before run()")
        _require(not args, "positional arguments after paged_kv_cache are not supported")
        _require(tuple(q.shape) == (self._B, self._Hq, self._D),
                 f"q must be [{self._B}, {self._Hq}, {self._D}]")
        k, v = self._kv(paged_kv_cache)
        if not return_lse:
            return paged_decode_attention(q, k, v, self._bt, self._sl, self._scale, self._S,
                                          out=out, workspace=self._ws_view)
        o_part, lse2 = paged_decode_attention_partial(q, k, v, self._bt, self._sl, self._scale,
                                                      self._S)
        o32 = torch.empty(self._B, self._Hq, self._D, dtype=torch.float32, device=q.device)
        l32 = lse if lse is not None else torch.empty(self._B, self._Hq, dtype=torch.float32,
                                                      device=q.device)
        merge_states_into(o_part, lse2, o32, l32)
        if out is None:
            out = torch.empty_like(q)
        out.copy_(o32)
        return out, l32

    forward = run


__all__ = ["BatchDecodeWithPagedKVCacheWrapper", "csr_to_block_table", "BptArgumentError"]
