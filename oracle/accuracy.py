"""Synthetic accuracy of the KIVI formats, in numpy float64. TEST INFRASTRUCTURE ONLY.

The reference keeps accuracy (perplexity, needle-in-a-haystack) separate from speed
(README.md:90) and has no quantized path. Perplexity needs model weights; these checks need
none. They measure what a format does to attention itself, on the BASELINE KIVI distribution
(K ~ N(0, 1) with 4 seeded x10 outlier channels per kv head, V ~ N(0, 1), block_size 64):

* needle in a haystack: one token's key is planted along the mean direction of its kv head's
  group of queries, scaled so that for a typical head of the group it takes about half of the
  softmax mass (its score sits at the haystack's log-sum-exp). The needle weight is its softmax
  weight, per q head; a format must recover it: |w_fmt - w_fp16| / w_fp16;
* output error against the unquantized fp16 cache: per q head ||o_fmt - o_fp16|| / ||o_fp16||
  (relative RMS) and the largest absolute difference.

All attention here is float64 on the fp16 cache or on the cache dequantized by the numpy
specification (oracle.kivi), i.e. the error of the format, not of any kernel.
"""
import numpy as np

from oracle import kivi
from oracle.cache import rng

HQ, HKV, D, BS = 32, 8, 128, 64


def needle_case(seed: int, ctx: int, outlier_channels: int = 4, outlier_scale: float = 10.0,
                Hq: int = HQ, Hkv: int = HKV, Dh: int = D):
    """q [Hq, D], k, v [ctx, Hkv, D] (fp16) and the needle position.

    The haystack follows the BASELINE KIVI distribution; the needle key of kv head h is
    a * u_h, u_h the unit mean direction of the group's queries, with a chosen so that the
    needle's score equals the group's mean haystack log-sum-exp."""
    g = rng(seed)
    q = g.standard_normal((Hq, Dh), dtype=np.float32).astype(np.float16)
    k = g.standard_normal((ctx, Hkv, Dh), dtype=np.float32)
    for h in range(Hkv):
        ch = g.choice(Dh, size=outlier_channels, replace=False)
        k[:, h, ch] *= np.float32(outlier_scale)
    k = k.astype(np.float16)
    v = g.standard_normal((ctx, Hkv, Dh), dtype=np.float32).astype(np.float16)
    pos = int(g.integers(ctx // 8, ctx - ctx // 8))
    group = Hq // Hkv
    qf = q.astype(np.float64).reshape(Hkv, group, Dh)
    scale = 1.0 / np.sqrt(Dh)
    for h in range(Hkv):
        u = qf[h].sum(axis=0)
        u /= np.linalg.norm(u)
        s = (k[:, h].astype(np.float64) @ qf[h].T) * scale         # [ctx, group]
        lse = np.log(np.exp(s - s.max(0)).sum(0)) + s.max(0)
        a = lse.mean() / ((qf[h] @ u).mean() * scale)
        k[pos, h] = (a * u).astype(np.float16)
    return q, k, v, pos


def quantized_kv(k: np.ndarray, v: np.ndarray, fmt: str, block_size: int = BS):
    """k, v [n, H, D] fp16 -> the float32 K, V [n, H, D] a KIVI cache of them dequantizes to."""
    n, H, Dh = k.shape
    pages = (n + block_size - 1) // block_size
    bt = np.arange(pages, dtype=np.int32)[None]
    cache = kivi.empty_cache(pages, block_size, H, Dh, fmt)
    kivi.quantize_append(cache, k[None], v[None], [n], [0], bt, block_size, fmt)
    kd, vd = kivi.dequantize_cache(cache, fmt)
    return kd.reshape(-1, H, Dh)[:n], vd.reshape(-1, H, Dh)[:n]


def attention64(q: np.ndarray, k: np.ndarray, v: np.ndarray, pos: int):
    """float64 attention of q [Hq, D] over k, v [n, Hkv, D]: (out [Hq, D], needle weight [Hq])."""
    Hq, Dh = q.shape
    Hkv = k.shape[1]
    group = Hq // Hkv
    qf = q.astype(np.float64).reshape(Hkv, group, Dh)
    kf = k.astype(np.float64).transpose(1, 0, 2)
    vf = v.astype(np.float64).transpose(1, 0, 2)
    s = np.matmul(qf, kf.transpose(0, 2, 1)) / np.sqrt(Dh)          # [Hkv, group, n]
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    return np.matmul(p, vf).reshape(Hq, Dh), p[..., pos].reshape(Hq)


def format_accuracy(seed: int, ctx: int, fmt: str, **kw):
    """Needle recovery and output error of one format against the fp16 cache."""
    q, k, v, pos = needle_case(seed, ctx, **kw)
    o16, w16 = attention64(q, k, v, pos)
    kd, vd = quantized_kv(k, v, fmt)
    oq, wq = attention64(q, kd, vd, pos)
    rel_rms = np.linalg.norm(oq - o16, axis=1) / np.linalg.norm(o16, axis=1)
    return {"ctx": ctx, "fmt": fmt, "needle_pos": pos,
            "needle_weight_fp16": w16, "needle_weight": wq,
            "needle_rel_err": float(np.max(np.abs(wq - w16) / w16)),
            "out_rel_rms": float(rel_rms.max()), "out_rel_rms_mean": float(rel_rms.mean()),
            "out_max_abs": float(np.abs(oq - o16).max())}
