"""numpy fp32 restatement of the reference oracle. TEST INFRASTRUCTURE ONLY.

Follows ``paged_decode_attention_ref`` in src/bpt/reference.py:20-49 step by step:

  * per sequence b: n = seq_lens[b], n_blocks = ceil(n / block_size)      (reference.py:37-38)
  * gather the first n_blocks physical pages named by block_table[b]     (reference.py:39)
  * flatten to [n_blocks*block_size, Hkv, D] and drop the tail past n    (reference.py:41-42)
  * fp32 math; q head h reads kv head h // group                         (reference.py:43-45)
  * scores = q . k * scale, softmax over n, probs . v                     (reference.py:46-48)
  * cast the result back to q.dtype                                       (reference.py:48)

The GQA expansion (``repeat_interleave``) is expressed as a reshape of q to
[Hkv, group, D] so each kv head is multiplied once by its group of q heads; this is the same
arithmetic (fp32 products and sums), just without materialising the 4x copy.

An empty sequence (n == 0) yields zeros, which is what the reference's einsum over an empty
token axis returns.
"""
import math
from typing import Optional

import numpy as np


def _softmax_rows(scores: np.ndarray) -> np.ndarray:
    """torch.softmax(x, -1): exp(x - max) / sum, in fp32 (reference.py:47)."""
    m = scores.max(axis=-1, keepdims=True)
    e = np.exp(scores - m, dtype=np.float32)
    return e / e.sum(axis=-1, keepdims=True, dtype=np.float32)


def attend_one(q_b: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """One sequence: q_b [Hq, D], k/v [n, Hkv, D] (any float dtype) -> fp32 [Hq, D]."""
    Hq, D = q_b.shape
    n, Hkv, _ = k.shape
    group = Hq // Hkv
    if n == 0:
        return np.zeros((Hq, D), dtype=np.float32)
    qf = q_b.astype(np.float32).reshape(Hkv, group, D)
    kf = np.ascontiguousarray(k.astype(np.float32).transpose(1, 0, 2))  # [Hkv, n, D]
    vf = np.ascontiguousarray(v.astype(np.float32).transpose(1, 0, 2))
    scores = np.matmul(qf, kf.transpose(0, 2, 1)) * np.float32(scale)  # [Hkv, group, n]
    probs = _softmax_rows(scores.astype(np.float32))
    out = np.matmul(probs, vf)  # [Hkv, group, D]
    return out.reshape(Hq, D).astype(np.float32)


def gather_sequence(k_cache: np.ndarray, block_table: np.ndarray, b: int, n: int) -> np.ndarray:
    """Pages of sequence b flattened to [n, Hkv, D] (reference.py:38-42)."""
    _, bs, Hkv, D = k_cache.shape
    nb = (n + bs - 1) // bs
    blocks = block_table[b, :nb].astype(np.int64)
    return k_cache[blocks].reshape(-1, Hkv, D)[:n]


def paged_decode_attention_ref(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
                               block_table: np.ndarray, seq_lens: np.ndarray,
                               scale: Optional[float] = None,
                               out_dtype=None) -> np.ndarray:
    """Oracle: q [B, Hq, D], caches [num_blocks, block_size, Hkv, D] -> [B, Hq, D].

    The caches may be fp16 (the FP16 path) or fp32 (a KIVI cache dequantized by
    ``oracle.kivi``); math is fp32 either way and the result is cast to ``out_dtype``
    (default q.dtype), as reference.py:35,48 casts to q.dtype.
    """
    B, Hq, D = q.shape
    _, _, Hkv, _ = k_cache.shape
    assert Hq % Hkv == 0, "q heads must be a multiple of kv heads"
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    out = np.empty((B, Hq, D), dtype=out_dtype or q.dtype)
    for b in range(B):
        n = int(seq_lens[b])
        k = gather_sequence(k_cache, block_table, b, n)
        v = gather_sequence(v_cache, block_table, b, n)
        out[b] = attend_one(q[b], k, v, scale).astype(out.dtype)
    return out


def paged_decode_attention_partial(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
                                   block_table: np.ndarray, seq_lens: np.ndarray,
                                   token_lo: np.ndarray, token_hi: np.ndarray,
                                   scale: Optional[float] = None):
    """Normalised partial attention over tokens [token_lo[b], token_hi[b]) of each sequence.

    Returns (o [B, Hq, D] fp32, lse [B, Hq] fp32, natural log). An empty range gives o = 0 and
    lse = -inf. This is the per-split state of the reference's split kernel
    (src/bpt/triton_fp16.py:138-144) and the per-rank state of sequence sharding; merging
    states with w = exp(lse - max lse) (triton_fp16.py:152-162) gives the full result.
    """
    B, Hq, D = q.shape
    _, _, Hkv, _ = k_cache.shape
    group = Hq // Hkv
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    o = np.zeros((B, Hq, D), dtype=np.float32)
    lse = np.full((B, Hq), -np.inf, dtype=np.float32)
    for b in range(B):
        n = int(seq_lens[b])
        lo, hi = int(token_lo[b]), min(int(token_hi[b]), n)
        if hi <= lo:
            continue
        k = gather_sequence(k_cache, block_table, b, n)[lo:hi]
        v = gather_sequence(v_cache, block_table, b, n)[lo:hi]
        qf = q[b].astype(np.float32).reshape(Hkv, group, D)
        kf = k.astype(np.float32).transpose(1, 0, 2)
        vf = v.astype(np.float32).transpose(1, 0, 2)
        s = np.matmul(qf, kf.transpose(0, 2, 1)) * np.float32(scale)
        m = s.max(axis=-1, keepdims=True)
        e = np.exp(s - m)
        l = e.sum(axis=-1, keepdims=True)
        o[b] = (np.matmul(e, vf) / l).reshape(Hq, D)
        lse[b] = (m + np.log(l)).reshape(Hq)
    return o, lse


def merge_states(o_parts, lse_parts):
    """LSE-weighted merge of partial states (reference: src/bpt/triton_fp16.py:147-163).

    o_parts [P, ..., D], lse_parts [P, ...] -> merged o [..., D] fp32. All-empty -> 0.
    """
    o_parts = np.asarray(o_parts, dtype=np.float32)
    lse_parts = np.asarray(lse_parts, dtype=np.float32)
    mx = lse_parts.max(axis=0)
    safe = np.where(np.isfinite(mx), mx, 0.0).astype(np.float32)
    w = np.exp(lse_parts - safe[None])
    den = w.sum(axis=0)
    num = (w[..., None] * o_parts).sum(axis=0)
    return np.where(den[..., None] > 0, num / np.where(den > 0, den, 1.0)[..., None], 0.0)
