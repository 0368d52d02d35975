"""What a KIVI format does to attention, measured through the decode kernels (no model needed).

The reference keeps accuracy checks (perplexity, needle-in-a-haystack; README.md:90) apart from
speed, and has no quantized path. Perplexity needs model weights; this study needs none. On
synthetic inputs with the BASELINE KIVI distribution (K ~ N(0, 1) with 4 seeded x10 outlier
channels per kv head, V ~ N(0, 1), block_size 64) it plants a needle and reports, per format:

* the needle's attention weight per q head, recovered through the decode kernel: two decodes
  whose caches differ only in the needle token's value give o_1 - o_2 = w (v^_1 - v^_2), so
  w = (o_1 - o_2) . (v^_1 - v^_2) / |v^_1 - v^_2|^2 (v^ = the stored value, dequantized); the
  same measurement on the fp16 cache gives the unquantized weight;
* the output error of the format against the fp16 cache (both decoded by bpt's kernels):
  per q head ||o_fmt - o_fp16|| / ||o_fp16|| and the largest absolute difference.

The needle key of kv head h is a * u_h, u_h the unit mean direction of the group's queries,
with a set so that its score equals the group's mean haystack log-sum-exp: about half the
softmax mass for a typical head of the group.
"""
import math
from typing import Optional

import torch

from .decode import paged_decode_attention
from .quant import empty_kivi_cache, paged_decode_attention_kivi, quantize_append

HQ, HKV, D = 32, 8, 128


def needle_inputs(ctx: int, seed: int = 0, device="cuda", outlier_channels: int = 4,
                  outlier_scale: float = 10.0, q_heads: int = HQ, kv_heads: int = HKV,
                  head_dim: int = D):
    """(q [Hq, D], k, v [ctx, Hkv, D] fp16, needle position) generated on ``device``."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    dg = torch.Generator(device=device).manual_seed(seed + 1)
    q = torch.randn(q_heads, head_dim, generator=dg, device=device).to(torch.float16)
    mult = torch.ones(kv_heads, head_dim)
    for h in range(kv_heads):
        mult[h, torch.randperm(head_dim, generator=g)[:outlier_channels]] = outlier_scale
    k = torch.randn(ctx, kv_heads, head_dim, generator=dg, device=device) * mult.to(device)
    k = k.to(torch.float16)
    v = torch.randn(ctx, kv_heads, head_dim, generator=dg, device=device).to(torch.float16)
    pos = int(torch.randint(ctx // 8, ctx - ctx // 8, (1,), generator=g))
    group = q_heads // kv_heads
    qf = q.double().reshape(kv_heads, group, head_dim)
    scale = 1.0 / math.sqrt(head_dim)
    for h in range(kv_heads):
        u = qf[h].sum(0)
        u = u / u.norm()
        s = (k[:, h].double() @ qf[h].T) * scale                       # [ctx, group]
        lse = torch.logsumexp(s, dim=0)
        a = lse.mean() / ((qf[h] @ u).mean() * scale)
        k[pos, h] = (a * u).to(torch.float16)
    return q, k, v, pos


def _paged(x: torch.Tensor, block_size: int) -> torch.Tensor:
    """[n, H, D] -> a paged cache [pages, block_size, H, D] (zero-padded last page)."""
    n, H, Dh = x.shape
    pages = (n + block_size - 1) // block_size
    out = torch.zeros(pages * block_size, H, Dh, dtype=x.dtype, device=x.device)
    out[:n] = x
    return out.view(pages, block_size, H, Dh)


def _needle_value(cache, pos: int) -> torch.Tensor:
    """The dequantized value of token ``pos`` (its page is pos // block_size): [Hkv, D] fp64."""
    bs = cache.block_size
    page, slot = pos // bs, pos % bs
    vs = cache.v_scale[page, slot].double()[:, None]
    if cache.fmt == "int4":
        row = cache.v_codes[page, slot // 2]
        codes = (row >> 4) if slot % 2 else (row & 0xF)
    else:
        codes = cache.v_codes[page, slot]
    if cache.fmt == "fp8":
        return codes.view(torch.float8_e4m3fn).double() * vs
    return codes.double() * vs + cache.v_zero[page, slot].double()[:, None]


def _weights(o1, o2, dv, q_heads, kv_heads):
    """w per q head from two outputs and the needle's value difference [Hkv, D]."""
    group = q_heads // kv_heads
    d = (o1.double() - o2.double()).view(kv_heads, group, -1)
    return ((d * dv[:, None]).sum(-1) / (dv * dv).sum(-1)[:, None]).reshape(q_heads)


def needle_study(fmt: str, ctx: int, seed: int = 0, device="cuda", block_size: int = 64,
                 num_splits: Optional[int] = None, inputs=None) -> dict:
    """Needle recovery and output error of ``fmt`` ("int8", "fp8", "int4") against the fp16
    cache, at one context length. Tensors in the result are on the CPU."""
    q, k, v, pos = inputs if inputs is not None else needle_inputs(ctx, seed, device)
    dev = q.device
    Hkv = k.shape[1]
    v2 = v.clone()
    v2[pos] = -v[pos]
    pages = (ctx + block_size - 1) // block_size
    bt = torch.arange(pages, dtype=torch.int32, device=dev)[None]
    sl = torch.tensor([ctx], dtype=torch.int32, device=dev)
    qb = q[None]
    kc = _paged(k, block_size)
    o16 = [paged_decode_attention(qb, kc, _paged(vv, block_size), bt, sl,
                                  num_splits=num_splits)[0] for vv in (v, v2)]
    caches = []
    for vv in (v, v2):
        cache = empty_kivi_cache(pages, block_size, Hkv, q.shape[1], fmt, device=dev)
        quantize_append(cache, k[None], vv[None], sl, torch.zeros_like(sl), bt)
        caches.append(cache)
    oq = [paged_decode_attention_kivi(qb, c, bt, sl, num_splits=num_splits)[0] for c in caches]
    w16 = _weights(o16[0], o16[1], (v[pos].double() - v2[pos].double()), q.shape[0], Hkv)
    dvq = _needle_value(caches[0], pos) - _needle_value(caches[1], pos)
    wq = _weights(oq[0], oq[1], dvq, q.shape[0], Hkv)
    diff = oq[0].double() - o16[0].double()
    rel_rms = diff.norm(dim=-1) / o16[0].double().norm(dim=-1)
    return {"fmt": fmt, "ctx": ctx, "needle_pos": pos,
            "needle_weight_fp16": w16.cpu(), "needle_weight": wq.cpu(),
            "needle_rel_err": float(((wq - w16).abs() / w16).max()),
            "needle_rel_err_median": float(((wq - w16).abs() / w16).median()),
            "out_rel_rms": float(rel_rms.max()), "out_rel_rms_mean": float(rel_rms.mean()),
            "out_max_abs": float(diff.abs().max()),
            "outputs": {"fp16": o16[0].cpu(), fmt: oq[0].cpu()}}


def summarize(r: dict) -> dict:
    """The scalar figures of a ``needle_study`` result (for a JSON line)."""
    w16 = r["needle_weight_fp16"]
    return {"needle_weight_fp16_median": float(w16.median()),
            "needle_weight_median": float(r["needle_weight"].median()),
            "needle_rel_err_max": r["needle_rel_err"],
            "needle_rel_err_median": r["needle_rel_err_median"],
            "out_rel_rms_max": r["out_rel_rms"], "out_rel_rms_mean": r["out_rel_rms_mean"],
            "out_max_abs": r["out_max_abs"]}


__all__ = ["needle_inputs", "needle_study", "summarize"]
