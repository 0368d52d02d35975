"""Seeded numpy builders for paged KV caches. TEST INFRASTRUCTURE ONLY.

``build_paged_cache`` follows src/bpt/reference.py:52-82: contiguous k/v [B, S, Hkv, D] are
scattered into physical pages through a random permutation, and every slot that no sequence
owns is filled with large garbage (100 * N(0,1)) so block-table and masking bugs cannot pass
by accident. Two table modes:

  "reference"  num_blocks = B * max_blocks and the whole table is one permutation
               (reference.py:65-67)
  "spare"      num_blocks = sum(ceil(n/bs)) + spare; each sequence's first ceil(n/bs) entries
               come from one permutation of the physical ids and the rest of the row is 0
               (the BASELINE CPU-correctness configuration)

All randomness comes from ``numpy.random.Generator(PCG64(seed))`` so the GPU box regenerates
bit-identical inputs from the seed; golden fixtures store a digest of the inputs to prove it.
"""
import hashlib
from typing import Optional, Sequence

import numpy as np


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def normal_f16(g: np.random.Generator, shape, scale: float = 1.0) -> np.ndarray:
    x = g.standard_normal(size=shape, dtype=np.float32)
    if scale != 1.0:
        x *= np.float32(scale)
    return x.astype(np.float16)


def make_qkv(g: np.random.Generator, lens: Sequence[int], Hq: int, Hkv: int, D: int,
             outlier_channels: int = 0, outlier_scale: float = 10.0):
    """q [B, Hq, D], k, v [B, max(lens), Hkv, D] fp16, all N(0, 1).

    ``outlier_channels`` > 0 scales that many seeded key channels per kv head by
    ``outlier_scale`` (the KIVI workload: 4 outlier channels x10).
    """
    B, S = len(lens), max(max(lens), 1)
    q = normal_f16(g, (B, Hq, D))
    k = g.standard_normal(size=(B, S, Hkv, D), dtype=np.float32)
    if outlier_channels:
        for h in range(Hkv):
            ch = g.choice(D, size=outlier_channels, replace=False)
            k[:, :, h, ch] *= np.float32(outlier_scale)
    k = k.astype(np.float16)
    v = normal_f16(g, (B, S, Hkv, D))
    return q, k, v


def block_table_for(g: np.random.Generator, lens: Sequence[int], block_size: int,
                    mode: str = "reference", spare: int = 64,
                    max_blocks: Optional[int] = None):
    """(block_table [B, max_blocks] int32, num_blocks)."""
    B = len(lens)
    pages = [(int(n) + block_size - 1) // block_size for n in lens]
    mb = max(max(pages), 1) if max_blocks is None else max_blocks
    if mode == "reference":
        num_blocks = B * mb
        bt = g.permutation(num_blocks).reshape(B, mb).astype(np.int32)
        return bt, num_blocks
    if mode == "spare":
        num_blocks = sum(pages) + spare
        perm = g.permutation(num_blocks).astype(np.int32)
        bt = np.zeros((B, mb), dtype=np.int32)
        off = 0
        for b, p in enumerate(pages):
            bt[b, :p] = perm[off:off + p]
            off += p
        return bt, num_blocks
    raise ValueError(mode)


def scatter_pages(x: np.ndarray, lens: Sequence[int], block_table: np.ndarray,
                  num_blocks: int, block_size: int, g: np.random.Generator,
                  garbage: float = 100.0) -> np.ndarray:
    """Contiguous x [B, S, Hkv, D] -> cache [num_blocks, block_size, Hkv, D] (reference.py:69-80)."""
    _, _, Hkv, D = x.shape
    cache = normal_f16(g, (num_blocks, block_size, Hkv, D), garbage) if garbage else \
        np.zeros((num_blocks, block_size, Hkv, D), dtype=x.dtype)
    cache = cache.astype(x.dtype)
    for b, n in enumerate(lens):
        n = int(n)
        for i in range((n + block_size - 1) // block_size):
            lo, hi = i * block_size, min((i + 1) * block_size, n)
            cache[int(block_table[b, i]), : hi - lo] = x[b, lo:hi]
    return cache


def build_paged_cache(k: np.ndarray, v: np.ndarray, lens: Sequence[int], block_size: int,
                      g: np.random.Generator, mode: str = "reference", spare: int = 64,
                      garbage: float = 100.0):
    """(k_cache, v_cache, block_table, num_blocks) — reference.py:52-82 semantics."""
    bt, nb = block_table_for(g, lens, block_size, mode, spare)
    kc = scatter_pages(k, lens, bt, nb, block_size, g, garbage)
    vc = scatter_pages(v, lens, bt, nb, block_size, g, garbage)
    return kc, vc, bt, nb


def ragged_lens(g: np.random.Generator, B: int, ctx: int, lo_frac: float = 0.75):
    """seq_len ~ U[lo_frac * ctx, ctx] (the BASELINE FP16 batch workload)."""
    return [int(x) for x in g.integers(int(lo_frac * ctx), ctx + 1, size=B)]


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()[:32]


def fp16_case(seed: int, lens: Sequence[int], Hq: int, Hkv: int, D: int, block_size: int,
              mode: str = "reference", spare: int = 64, garbage: float = 100.0):
    """The standard FP16 parity case: returns dict of numpy arrays + metadata."""
    g = rng(seed)
    q, k, v = make_qkv(g, lens, Hq, Hkv, D)
    kc, vc, bt, nb = build_paged_cache(k, v, lens, block_size, g, mode, spare, garbage)
    return dict(q=q, k_cache=kc, v_cache=vc, block_table=bt,
                seq_lens=np.asarray(lens, dtype=np.int32), num_blocks=nb)
