"""Multi-GPU decode over one node: batch sharding and sequence sharding (no reference
counterpart; the reference is single-GPU).

One process per GPU, ``torch.distributed`` with the NCCL backend over NVLink / NVSwitch.

* Batch sharding (B >= number of GPUs): each rank owns a contiguous slice of the sequences
  together with their KV pages and block-table rows, and decodes them locally. Sequences are
  independent, so there is no collective on the data path; ``gather_outputs`` optionally
  all-gathers the [B_local, Hq, D] outputs for a consumer that needs all of them.

* Sequence sharding (batch 1, long context): rank r owns the page-aligned token range
  ``token_shards(...)[r]`` of every sequence in its own KV pool. Each rank runs the split-KV
  kernel over its tokens and merges its splits into one fp32 state per (sequence, q head) --
  o [B, Hq, D] and its log2-sum-exp [B, Hq] -- packed into one flat buffer; one
  ``all_gather_into_tensor`` exchanges the states (B * Hq * (D + 1) * 4 bytes per rank, 16.5 KB
  at the Llama-3-8B shape and B=1) and every rank merges the gathered states with the
  reference's split-merge formula (src/bpt/triton_fp16.py:152-162) into the fp16 output.
  All ranks take the same collective steps in the same order; a rank that fails or never
  joins surfaces as the process group's timeout error on the others.

* Fused exchange (``SequenceShardExchange``): the same sequence sharding without a collective
  on the data path. Each rank maps the others' receive buffers once (CUDA IPC over NVLink);
  per call the split kernel is followed by one kernel (bpt_seqx_merge_fp16) that merges the
  splits, stores the rank's states straight into every peer's buffer, waits (time-bounded) for
  theirs and writes the merged output: two launches per call, capturable in a CUDA graph.
"""
import ctypes
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib
from .decode import _require, _stream_handle, merge_states_into, paged_decode_attention, \
    paged_decode_attention_partial


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous balanced [lo, hi) slice of n items for `rank` of `world`."""
    _require(world >= 1 and 0 <= rank < world, "bad world/rank")
    return (n * rank) // world, (n * (rank + 1)) // world


def token_shards(seq_len: int, block_size: int, world: int) -> List[Tuple[int, int]]:
    """Page-aligned token ranges [lo, hi) covering a sequence, one per rank (balanced by
    pages; a rank may get an empty range when there are fewer pages than ranks)."""
    pages = (int(seq_len) + block_size - 1) // block_size
    out = []
    for r in range(world):
        p0, p1 = shard_range(pages, world, r)
        out.append((min(p0 * block_size, seq_len), min(p1 * block_size, seq_len)))
    return out


_MERGE_RANKS = None


def _merge_ranks_fn():
    global _MERGE_RANKS
    if _MERGE_RANKS is None:
        _MERGE_RANKS = _lib.register("bpt_merge_rank_states", ctypes.c_int, [
            ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p])
    return _MERGE_RANKS


def state_buffer(batch: int, q_heads: int, head_dim: int, device) -> torch.Tensor:
    """Flat fp32 buffer holding one rank's state: o [B, Hq, D] then lse [B, Hq]."""
    return torch.empty(batch * q_heads * (head_dim + 1), dtype=torch.float32, device=device)


def split_state(buf: torch.Tensor, batch: int, q_heads: int, head_dim: int):
    n = batch * q_heads * head_dim
    return buf[:n].view(batch, q_heads, head_dim), buf[n:].view(batch, q_heads)


def merge_rank_states(gathered: torch.Tensor, ranks: int, batch: int, q_heads: int,
                      head_dim: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Merge `ranks` gathered state blocks [ranks * B*Hq*(D+1)] into fp16 [B, Hq, D]."""
    _require(gathered.is_cuda and gathered.dtype == torch.float32 and gathered.is_contiguous(),
             "gathered states must be a contiguous fp32 CUDA tensor")
    _require(gathered.numel() == ranks * batch * q_heads * (head_dim + 1),
             "gathered states have the wrong size")
    if out is None:
        out = torch.empty(batch, q_heads, head_dim, dtype=torch.float16, device=gathered.device)
    rc = _merge_ranks_fn()(gathered.data_ptr(), ranks, batch, q_heads, head_dim, out.data_ptr(),
                           out.stride(0), out.stride(1), _stream_handle(gathered.device))
    _lib.check(rc, "bpt_merge_rank_states")
    return out


def local_state(q: torch.Tensor, k_cache, v_cache, block_table: torch.Tensor,
                seq_lens: torch.Tensor, scale: Optional[float] = None,
                num_splits: Optional[int] = None, out_state: Optional[torch.Tensor] = None,
                kivi_cache=None) -> torch.Tensor:
    """This rank's merged fp32 state over its own tokens, packed for the all-gather.

    FP16 caches pass k_cache / v_cache; KIVI caches pass kivi_cache (k_cache = v_cache = None).
    """
    B, Hq, D = q.shape
    if kivi_cache is not None:
        from .quant import paged_decode_attention_kivi_partial
        o_part, lse = paged_decode_attention_kivi_partial(q, kivi_cache, block_table, seq_lens,
                                                          scale, num_splits)
    else:
        o_part, lse = paged_decode_attention_partial(q, k_cache, v_cache, block_table,
                                                     seq_lens, scale, num_splits)
    if out_state is None:
        out_state = state_buffer(B, Hq, D, q.device)
    o, l2 = split_state(out_state, B, Hq, D)
    merge_states_into(o_part, lse, o, l2)
    return out_state


_SEQX = None


def _seqx_fns():
    global _SEQX
    if _SEQX is None:
        c_vp, c_int = ctypes.c_void_p, ctypes.c_int
        _SEQX = dict(
            bytes=_lib.register("bpt_seqx_buffer_bytes", ctypes.c_size_t,
                                [c_int, c_int, c_int, c_int]),
            alloc=_lib.register("bpt_seqx_alloc", c_int,
                                [ctypes.c_size_t, ctypes.POINTER(c_vp), c_vp]),
            open=_lib.register("bpt_seqx_open", c_int, [c_vp, ctypes.POINTER(c_vp)]),
            close=_lib.register("bpt_seqx_close", c_int, [c_vp]),
            free=_lib.register("bpt_seqx_free", c_int, [c_vp]),
            merge=_lib.register("bpt_seqx_merge_fp16", c_int, [
                c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp, c_int, c_int, c_vp,
                ctypes.c_int64, ctypes.c_int64, c_vp, ctypes.c_uint, c_vp]))
    return _SEQX


IPC_HANDLE_BYTES = 64


class SequenceShardExchange:
    """Receive buffers of a sequence-sharded decode group, mapped into every rank over NVLink.

    Build it once per process group and shape (all ranks, same arguments); it all-gathers the
    64-byte CUDA IPC handles of the ranks' buffers over `group` and maps the peers' buffers.
    ``merge(o_part, lse, out)`` then runs the fused split merge + exchange + rank merge kernel.
    The kernels of the ranks wait on each other (time-bounded by ``budget_us``), so every rank
    must issue the same calls in the same order. ``close()`` unmaps and frees the buffers.
    """

    def __init__(self, batch: int, q_heads: int, head_dim: int, group=None, device=None,
                 budget_us: int = 2_000_000):
        f = _seqx_fns()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        _require(1 <= self.world <= 8, "the fused exchange serves 1 to 8 ranks")
        _require(head_dim % 4 == 0 and head_dim <= 256, "head_dim must be a multiple of 4, <= 256")
        self.batch, self.q_heads, self.head_dim = batch, q_heads, head_dim
        self.budget_us = int(budget_us)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        nbytes = f["bytes"](self.world, batch, q_heads, head_dim)
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * IPC_HANDLE_BYTES)()
        _lib.check(f["alloc"](nbytes, ctypes.byref(own), ctypes.cast(handle, ctypes.c_void_p)),
                   "bpt_seqx_alloc")
        self._own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        ptrs, self._opened = [], []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(self._own)
                continue
            p = ctypes.c_void_p()
            hb = (ctypes.c_char * IPC_HANDLE_BYTES).from_buffer_copy(h)
            _lib.check(f["open"](ctypes.cast(hb, ctypes.c_void_p), ctypes.byref(p)),
                       "bpt_seqx_open")
            ptrs.append(p.value)
            self._opened.append(p.value)
        self._ptrs = (ctypes.c_void_p * self.world)(*ptrs)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def merge(self, o_part: torch.Tensor, lse: torch.Tensor,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """o_part [B, Hq, S, D] / lse [B, Hq, S] of this rank -> merged fp16 [B, Hq, D]."""
        B, Hq, S, D = o_part.shape
        _require((B, Hq, D) == (self.batch, self.q_heads, self.head_dim),
                 "o_part shape does not match the exchange")
        _require(o_part.is_contiguous() and lse.is_contiguous(), "partials must be contiguous")
        if out is None:
            out = torch.empty(B, Hq, D, dtype=torch.float16, device=o_part.device)
        rc = _seqx_fns()["merge"](o_part.data_ptr(), lse.data_ptr(), B, Hq, D, S,
                                  ctypes.cast(self._ptrs, ctypes.c_void_p), self.world,
                                  self.rank, out.data_ptr(), out.stride(0), out.stride(1),
                                  self.status.data_ptr(), self.budget_us,
                                  _stream_handle(o_part.device))
        _lib.check(rc, "bpt_seqx_merge_fp16")
        return out

    def close(self):
        f = _seqx_fns()
        for p in self._opened:
            f["close"](p)
        self._opened = []
        if self._own:
            f["free"](self._own)
            self._own = None


def decode_sequence_sharded(q: torch.Tensor, k_cache, v_cache, block_table: torch.Tensor,
                            seq_lens: torch.Tensor, scale: Optional[float] = None,
                            num_splits: Optional[int] = None, *, group=None, kivi_cache=None,
                            out: Optional[torch.Tensor] = None,
                            exchange: Optional[SequenceShardExchange] = None) -> torch.Tensor:
    """Decode sequences whose tokens are spread over the ranks of `group`.

    Every rank passes the same q [B, Hq, D] and ITS OWN pages: block_table / seq_lens describe
    the rank's token range of each sequence (seq_lens[b] = tokens this rank holds, may be 0).
    Returns the full fp16 [B, Hq, D] result on every rank. With `exchange` the states move by
    the fused NVLink kernel (no collective, no host synchronisation); otherwise by one NCCL
    all-gather.
    """
    if exchange is not None:
        if kivi_cache is not None:
            from .quant import paged_decode_attention_kivi_partial
            o_part, lse = paged_decode_attention_kivi_partial(q, kivi_cache, block_table,
                                                              seq_lens, scale, num_splits)
        else:
            o_part, lse = paged_decode_attention_partial(q, k_cache, v_cache, block_table,
                                                         seq_lens, scale, num_splits)
        return exchange.merge(o_part, lse, out=out)
    world = dist.get_world_size(group)
    B, Hq, D = q.shape
    send = local_state(q, k_cache, v_cache, block_table, seq_lens, scale, num_splits,
                       kivi_cache=kivi_cache)
    recv = torch.empty(world * send.numel(), dtype=torch.float32, device=q.device)
    dist.all_gather_into_tensor(recv, send, group=group)
    return merge_rank_states(recv, world, B, Hq, D, out=out)


def decode_batch_sharded(q_local: torch.Tensor, k_cache, v_cache, block_table: torch.Tensor,
                         seq_lens: torch.Tensor, scale: Optional[float] = None,
                         num_splits: Optional[int] = None, *, kivi_cache=None,
                         out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Decode this rank's slice of the batch (its own sequences, pages and table rows).
    No communication: batch sharding needs none."""
    if kivi_cache is not None:
        from .quant import paged_decode_attention_kivi
        return paged_decode_attention_kivi(q_local, kivi_cache, block_table, seq_lens, scale,
                                           num_splits, out=out)
    return paged_decode_attention(q_local, k_cache, v_cache, block_table, seq_lens, scale,
                                  num_splits, out=out)


def gather_outputs(out_local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather equal-sized [B_local, Hq, D] outputs of a batch-sharded decode."""
    world = dist.get_world_size(group)
    res = torch.empty((world * out_local.shape[0],) + tuple(out_local.shape[1:]),
                      dtype=out_local.dtype, device=out_local.device)
    dist.all_gather_into_tensor(res, out_local.contiguous(), group=group)
    return res


__all__ = ["shard_range", "token_shards", "state_buffer", "split_state", "merge_rank_states",
           "local_state", "SequenceShardExchange", "decode_sequence_sharded",
           "decode_batch_sharded", "gather_outputs"]
