"""KIVI-quantized paged KV caches: INT8, FP8-E4M3 and INT4 (no reference counterpart).

The reference lists quantized KV as "not started"; this module implements the format the
BASELINE configurations describe. Keys are quantized per (page, kv head, channel) over the
page's tokens, values per (token, kv head) over the channels; INT8 / INT4 are asymmetric
(fp16 scale + zero-point), FP8-E4M3 symmetric (fp16 scale). Codes are bit-exact with the
numpy specification (oracle/kivi.py). Layout (bs = block_size, H kv heads, D head dim):

    INT8 / FP8  k_codes, v_codes [num_blocks, bs, H, D]  uint8
    INT4        k_codes [num_blocks, bs, H, D/2]  low nibble = even channel
                v_codes [num_blocks, bs/2, H, D]  low nibble = even token
    k_scale, k_zero [num_blocks, H, D] fp16;  v_scale, v_zero [num_blocks, bs, H] fp16

``quantize_append`` writes whole pages from fp16 rows (the cache-append step);
``paged_decode_attention_kivi`` is the fused-dequant decode over such a cache.
"""
import ctypes
import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from .decode import _require, _sm_count, _stream_handle, check_device_flags, CHECKS

FORMATS = {"int8": 1, "fp8": 2, "int4": 3}
c_i32, c_i64, c_vp = ctypes.c_int, ctypes.c_int64, ctypes.c_void_p


class KiviCacheC(ctypes.Structure):
    """Mirror of ``bpt_kivi_cache`` (include/bpt.h)."""
    _fields_ = [("format", c_i32), ("block_size", c_i32), ("kv_heads", c_i32),
                ("head_dim", c_i32), ("num_blocks", c_i64),
                ("k_codes", c_vp), ("k_codes_stride", c_i64 * 3),
                ("v_codes", c_vp), ("v_codes_stride", c_i64 * 3),
                ("k_scale", c_vp), ("k_zero", c_vp), ("k_param_stride", c_i64 * 2),
                ("v_scale", c_vp), ("v_zero", c_vp), ("v_param_stride", c_i64 * 2)]


@dataclass
class KiviCache:
    fmt: str
    block_size: int
    k_codes: torch.Tensor
    v_codes: torch.Tensor
    k_scale: torch.Tensor
    v_scale: torch.Tensor
    k_zero: Optional[torch.Tensor] = None
    v_zero: Optional[torch.Tensor] = None

    @property
    def num_blocks(self) -> int:
        return self.k_codes.shape[0]

    @property
    def kv_heads(self) -> int:
        return self.k_codes.shape[2]

    @property
    def head_dim(self) -> int:
        return self.v_codes.shape[3]

    @property
    def device(self) -> torch.device:
        return self.k_codes.device

    def tensors(self):
        return {k: getattr(self, k) for k in ("k_codes", "v_codes", "k_scale", "v_scale",
                                              "k_zero", "v_zero") if getattr(self, k) is not None}

    def validate(self):
        fmt, bs = self.fmt, self.block_size
        _require(fmt in FORMATS, f"unknown KIVI format {fmt!r}")
        nb, H, D = self.num_blocks, self.kv_heads, self.head_dim
        kd = D // 2 if fmt == "int4" else D
        vt = bs // 2 if fmt == "int4" else bs
        _require(self.k_codes.shape == (nb, bs, H, kd) and self.k_codes.dtype == torch.uint8,
                 f"k_codes must be uint8 {(nb, bs, H, kd)}")
        _require(self.v_codes.shape == (nb, vt, H, D) and self.v_codes.dtype == torch.uint8,
                 f"v_codes must be uint8 {(nb, vt, H, D)}")
        for name, shape in (("k_scale", (nb, H, D)), ("v_scale", (nb, bs, H))):
            t = getattr(self, name)
            _require(t.shape == shape and t.dtype == torch.float16, f"{name} must be fp16 {shape}")
        if fmt != "fp8":
            for name, shape in (("k_zero", (nb, H, D)), ("v_zero", (nb, bs, H))):
                t = getattr(self, name)
                _require(t is not None and t.shape == shape and t.dtype == torch.float16,
                         f"{name} must be fp16 {shape}")
        _require(self.k_codes.stride(3) == 1 and self.v_codes.stride(3) == 1,
                 "code arrays need a unit inner stride")
        _require(self.k_scale.stride(2) == 1 and self.v_scale.stride(2) == 1,
                 "scale arrays need a unit inner stride")
        if fmt != "fp8":
            _require(self.k_zero.stride() == self.k_scale.stride() and
                     self.v_zero.stride() == self.v_scale.stride(),
                     "zero-points must share the scales' strides")

    def to_c(self) -> KiviCacheC:
        self.validate()
        c = KiviCacheC()
        c.format = FORMATS[self.fmt]
        c.block_size = self.block_size
        c.kv_heads = self.kv_heads
        c.head_dim = self.head_dim
        c.num_blocks = self.num_blocks
        c.k_codes = self.k_codes.data_ptr()
        c.k_codes_stride[:] = list(self.k_codes.stride()[:3])
        c.v_codes = self.v_codes.data_ptr()
        c.v_codes_stride[:] = list(self.v_codes.stride()[:3])
        c.k_scale = self.k_scale.data_ptr()
        c.k_zero = self.k_zero.data_ptr() if self.k_zero is not None else None
        c.k_param_stride[:] = list(self.k_scale.stride()[:2])
        c.v_scale = self.v_scale.data_ptr()
        c.v_zero = self.v_zero.data_ptr() if self.v_zero is not None else None
        c.v_param_stride[:] = list(self.v_scale.stride()[:2])
        return c


def empty_kivi_cache(num_blocks: int, block_size: int, kv_heads: int, head_dim: int, fmt: str,
                     device="cuda") -> KiviCache:
    """Allocate a zeroed KIVI cache."""
    _require(fmt in FORMATS, f"unknown KIVI format {fmt!r}")
    _require(fmt != "int4" or (block_size % 2 == 0 and head_dim % 2 == 0),
             "INT4 needs even block_size and head_dim")
    kd = head_dim // 2 if fmt == "int4" else head_dim
    vt = block_size // 2 if fmt == "int4" else block_size
    z = lambda *s, dt: torch.zeros(*s, dtype=dt, device=device)  # noqa: E731
    return KiviCache(
        fmt=fmt, block_size=block_size,
        k_codes=z(num_blocks, block_size, kv_heads, kd, dt=torch.uint8),
        v_codes=z(num_blocks, vt, kv_heads, head_dim, dt=torch.uint8),
        k_scale=z(num_blocks, kv_heads, head_dim, dt=torch.float16),
        v_scale=z(num_blocks, block_size, kv_heads, dt=torch.float16),
        k_zero=None if fmt == "fp8" else z(num_blocks, kv_heads, head_dim, dt=torch.float16),
        v_zero=None if fmt == "fp8" else z(num_blocks, block_size, kv_heads, dt=torch.float16))


_APPEND = None


def _append_fn():
    global _APPEND
    if _APPEND is None:
        _APPEND = _lib.register("bpt_kivi_append", c_i32, [
            ctypes.POINTER(KiviCacheC), c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64,
            c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_i32, c_vp])
    return _APPEND


def quantize_append(cache: KiviCache, k_new: torch.Tensor, v_new: torch.Tensor,
                    new_lens: torch.Tensor, start_pos: torch.Tensor,
                    block_table: torch.Tensor) -> KiviCache:
    """Quantize tokens [start_pos[b], start_pos[b] + new_lens[b]) of each sequence into the cache.

    k_new / v_new [B, S, H, D] fp16 hold the new tokens from index 0; start_pos must be a
    multiple of block_size (pages are written whole). new_lens, start_pos, block_table are
    int32 device tensors. Runs on the current stream; no host synchronisation.
    """
    _require(k_new.dim() == 4 and k_new.shape == v_new.shape, "k_new/v_new must be [B, S, H, D]")
    B, S, H, D = k_new.shape
    _require(k_new.dtype == v_new.dtype == torch.float16, "k_new/v_new must be float16")
    _require(H == cache.kv_heads and D == cache.head_dim, "k_new shape does not match the cache")
    _require(k_new.stride(3) == 1 and v_new.stride(3) == 1, "k_new/v_new need a unit inner stride")
    for t, n in ((new_lens, "new_lens"), (start_pos, "start_pos"), (block_table, "block_table")):
        _require(t.dtype == torch.int32 and t.device == cache.device, f"{n} must be int32 on "
                 f"{cache.device}")
    _require(block_table.stride(1) == 1, "block_table rows must be contiguous")
    c = cache.to_c()
    rc = _append_fn()(ctypes.byref(c), k_new.data_ptr(), *k_new.stride()[:3], v_new.data_ptr(),
                      *v_new.stride()[:3], new_lens.data_ptr(), start_pos.data_ptr(),
                      block_table.data_ptr(), block_table.stride(0), block_table.shape[1], B, S,
                      _stream_handle(cache.device))
    _lib.check(rc, "bpt_kivi_append")
    return cache


_DECODE = None
_DECODE_PARTIAL = None


def _decode_fns():
    global _DECODE, _DECODE_PARTIAL
    if _DECODE is None:
        P = ctypes.POINTER(KiviCacheC)
        _DECODE = _lib.register("bpt_decode_kivi", c_i32, [
            P, c_vp, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp, c_i64, c_i64,
            c_i32, c_i32, c_i32, ctypes.c_float, c_i32, c_i32, c_vp, ctypes.c_size_t, c_vp])
        _DECODE_PARTIAL = _lib.register("bpt_decode_kivi_partial", c_i32, [
            P, c_vp, c_i64, c_i64, c_vp, c_i64, c_vp, c_i32, c_i32, c_i32, ctypes.c_float,
            c_i32, c_vp, c_vp, c_vp, c_vp])
    return _DECODE, _DECODE_PARTIAL


_SPLITS = None


def effective_splits_kivi(cache: "KiviCache", batch: int, q_heads: int, max_blocks: int,
                          num_splits: Optional[int], sm_count: int) -> int:
    """Split count a KIVI decode call uses (bpt_effective_splits_kivi): the kernel serving
    the format / group has its own tokens per stage and CTAs per SM."""
    global _SPLITS
    if _SPLITS is None:
        _SPLITS = _lib.register("bpt_effective_splits_kivi", c_i32, [c_i32] * 8)
    return int(_SPLITS(FORMATS[cache.fmt], batch, cache.kv_heads, q_heads, cache.block_size,
                       max_blocks, int(num_splits or 0), sm_count))


def _validate_decode(q, cache: KiviCache, block_table, seq_lens):
    _require(q.dim() == 3 and q.dtype == torch.float16 and q.stride(2) == 1,
             "q must be float16 [B, Hq, D] with unit inner stride")
    B, Hq, D = q.shape
    _require(D == cache.head_dim, "head_dim of q and cache differ")
    _require(Hq % cache.kv_heads == 0, "q heads must be a multiple of kv heads")
    _require(block_table.dim() == 2 and block_table.shape[0] == B and
             block_table.dtype == torch.int32 and block_table.stride(1) == 1,
             "block_table must be int32 [B, max_blocks] with contiguous rows")
    _require(seq_lens.shape == (B,) and seq_lens.dtype == torch.int32 and
             seq_lens.is_contiguous(), "seq_lens must be int32 [B]")
    dev = q.device
    _require(dev.type == "cuda", "bpt runs on CUDA tensors only (no CPU fallback)")
    for t, n in ((block_table, "block_table"), (seq_lens, "seq_lens"),
                 (cache.k_codes, "cache")):
        _require(t.device == dev, f"{n} is on {t.device}, q on {dev}")
    return B, Hq, D


def paged_decode_attention_kivi(q: torch.Tensor, cache: KiviCache, block_table: torch.Tensor,
                                seq_lens: torch.Tensor, scale: Optional[float] = None,
                                num_splits: Optional[int] = None, *,
                                out: Optional[torch.Tensor] = None,
                                workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """GQA decode over a KIVI-quantized paged cache (dequantization fused) -> [B, Hq, D] fp16.

    Same contract as ``bpt.paged_decode_attention`` (split semantics, no host sync, zeros for
    an empty sequence); matches fp32 attention on the dequantized cache.
    """
    from .decode import workspace_bytes
    B, Hq, D = _validate_decode(q, cache, block_table, seq_lens)
    dev = q.device
    sms = _sm_count(dev.index or 0)
    max_blocks = block_table.shape[1]
    S = effective_splits_kivi(cache, B, Hq, max_blocks, num_splits, sms)
    need = workspace_bytes(B, Hq, D, S)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    if CHECKS:
        workspace[:4].zero_()
    if out is None:
        out = torch.empty_like(q)
    c = cache.to_c()
    rc = _decode_fns()[0](ctypes.byref(c), q.data_ptr(), q.stride(0), q.stride(1),
                          block_table.data_ptr(), block_table.stride(0), seq_lens.data_ptr(),
                          out.data_ptr(), out.stride(0), out.stride(1), B, Hq, max_blocks,
                          float(scale if scale is not None else 1.0 / math.sqrt(D)),
                          int(num_splits or 0), sms, workspace.data_ptr(),
                          workspace.numel() * workspace.element_size(), _stream_handle(dev))
    _lib.check(rc, "bpt_decode_kivi")
    if CHECKS:
        check_device_flags(workspace, "bpt_decode_kivi")
    return out


def paged_decode_attention_kivi_partial(q: torch.Tensor, cache: KiviCache,
                                        block_table: torch.Tensor, seq_lens: torch.Tensor,
                                        scale: Optional[float] = None,
                                        num_splits: Optional[int] = None):
    """Stage 1 only over a KIVI cache: (o_part [B, Hq, S, D] fp32, lse [B, Hq, S] log2)."""
    B, Hq, D = _validate_decode(q, cache, block_table, seq_lens)
    dev = q.device
    S = effective_splits_kivi(cache, B, Hq, block_table.shape[1], num_splits,
                              _sm_count(dev.index or 0))
    o_part = torch.empty(B, Hq, S, D, dtype=torch.float32, device=dev)
    lse = torch.empty(B, Hq, S, dtype=torch.float32, device=dev)
    c = cache.to_c()
    rc = _decode_fns()[1](ctypes.byref(c), q.data_ptr(), q.stride(0), q.stride(1),
                          block_table.data_ptr(), block_table.stride(0), seq_lens.data_ptr(),
                          B, Hq, block_table.shape[1],
                          float(scale if scale is not None else 1.0 / math.sqrt(D)), S,
                          o_part.data_ptr(), lse.data_ptr(), None, _stream_handle(dev))
    _lib.check(rc, "bpt_decode_kivi_partial")
    return o_part, lse


def paged_decode_attention_kivi_with_residual(q: torch.Tensor, cache: KiviCache,
                                             block_table: torch.Tensor, seq_lens: torch.Tensor,
                                             k_res: torch.Tensor, v_res: torch.Tensor,
                                             res_lens: torch.Tensor,
                                             scale: Optional[float] = None,
                                             num_splits: Optional[int] = None, *,
                                             out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Decode over a KIVI cache whose newest tokens are still in full precision.

    The append quantizer writes whole pages, because key statistics are per page. A decode
    loop therefore keeps each sequence's not-yet-full last page in fp16 (KIVI's residual):
    k_res / v_res [B, R, Hkv, D] fp16 hold sequence b's res_lens[b] newest tokens (positions
    seq_lens[b] .. seq_lens[b] + res_lens[b] - 1; R a power of two >= 16, e.g. the page size).
    When a residual fills a page, the caller moves it into the cache with ``quantize_append``
    (start_pos = seq_lens[b], page-aligned) and empties it.

    The quantized pages and the residual are decoded by their own kernels into per-split
    partial softmax states. Those are merged in one pass (the split merge), so the result is
    attention over the union: the quantized part as fp32 math on the dequantized cache, the
    residual in fp16 as ``paged_decode_attention``.
    """
    from .decode import merge_partials, paged_decode_attention_partial
    B, Hq, D = _validate_decode(q, cache, block_table, seq_lens)
    _require(k_res.dim() == 4 and k_res.shape == v_res.shape and k_res.shape[0] == B and
             tuple(k_res.shape[2:]) == (cache.kv_heads, D) and
             k_res.dtype == v_res.dtype == torch.float16,
             "k_res / v_res must be float16 [B, R, Hkv, D] matching q and the cache")
    _require(res_lens.shape == (B,) and res_lens.dtype == torch.int32 and
             res_lens.device == q.device, "res_lens must be int32 [B] on q's device")
    R = k_res.shape[1]
    # the residual as a paged fp16 cache: one page of R tokens per sequence
    bt_res = torch.arange(B, dtype=torch.int32, device=q.device).view(B, 1)
    o_q, l_q = paged_decode_attention_kivi_partial(q, cache, block_table, seq_lens, scale,
                                                   num_splits)
    o_r, l_r = paged_decode_attention_partial(q, k_res, v_res, bt_res, res_lens, scale,
                                              max(1, min(4, R // 16)))
    return merge_partials(torch.cat([o_q, o_r], dim=2).contiguous(),
                          torch.cat([l_q, l_r], dim=2).contiguous(), out=out)


def random_kivi_workload(lens, q_heads: int, kv_heads: int, head_dim: int, block_size: int,
                         fmt: str, device, seed: int = 0, outlier_channels: int = 4,
                         outlier_scale: float = 10.0, spare_blocks: int = 0,
                         seqs_per_batch: int = 4):
    """Synthetic quantized decode inputs generated and quantized on ``device``.

    K ~ N(0, 1) with ``outlier_channels`` seeded channels per kv head scaled by
    ``outlier_scale``, V ~ N(0, 1), q ~ N(0, 1) (the BASELINE KIVI workload), quantized by the
    cache-append kernel a few sequences at a time. Returns dict(q, cache, block_table,
    seq_lens, num_blocks).
    """
    B = len(lens)
    pages = [(int(n) + block_size - 1) // block_size for n in lens]
    max_blocks = max(max(pages), 1)
    num_blocks = sum(pages) + spare_blocks
    g = torch.Generator(device="cpu").manual_seed(seed)
    perm = torch.randperm(num_blocks, generator=g)
    bt = torch.zeros(B, max_blocks, dtype=torch.int32)
    off = 0
    for b, p in enumerate(pages):
        bt[b, :p] = perm[off:off + p].to(torch.int32)
        off += p
    bt = bt.to(device)
    mult = torch.ones(kv_heads, head_dim)
    for h in range(kv_heads):
        ch = torch.randperm(head_dim, generator=g)[:outlier_channels]
        mult[h, ch] = outlier_scale
    mult = mult.to(device)
    cache = empty_kivi_cache(num_blocks, block_size, kv_heads, head_dim, fmt, device)
    dg = torch.Generator(device=device).manual_seed(seed + 1)
    q = torch.randn(B, q_heads, head_dim, generator=dg, device=device).to(torch.float16)
    for b0 in range(0, B, seqs_per_batch):
        sub = list(lens[b0:b0 + seqs_per_batch])
        S = max(max(sub), 1)
        k = torch.randn(len(sub), S, kv_heads, head_dim, generator=dg, device=device)
        k = (k * mult).to(torch.float16)
        v = torch.randn(len(sub), S, kv_heads, head_dim, generator=dg, device=device,
                        dtype=torch.float16)
        nl = torch.tensor(sub, dtype=torch.int32, device=device)
        quantize_append(cache, k, v, nl, torch.zeros_like(nl),
                        bt[b0:b0 + len(sub)].contiguous())
        del k, v
    return dict(q=q, cache=cache, block_table=bt,
                seq_lens=torch.tensor(list(lens), dtype=torch.int32, device=device),
                num_blocks=num_blocks)


__all__ = ["KiviCache", "KiviCacheC", "empty_kivi_cache", "quantize_append", "FORMATS",
           "paged_decode_attention_kivi", "paged_decode_attention_kivi_partial",
           "paged_decode_attention_kivi_with_residual",
           "effective_splits_kivi",
           "random_kivi_workload"]
