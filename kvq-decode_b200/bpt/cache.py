"""Paged-cache construction helpers (torch, any device).

``build_paged_cache`` keeps the reference's signature and semantics
(src/bpt/reference.py:52-82): contiguous k/v [B, S, Hkv, D] are scattered into randomly
permuted physical pages and every slot no sequence owns holds 100 * N(0, 1) garbage.

``random_paged_workload`` builds large synthetic decode workloads directly on the device
(the BASELINE configurations: q, K, V ~ N(0, 1) fp16, random-permutation block tables).
"""
from typing import Optional, Sequence, Tuple

import torch


def build_paged_cache(k: torch.Tensor, v: torch.Tensor, seq_lens: torch.Tensor,
                      block_size: int, generator: Optional[torch.Generator] = None
                      ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Scatter contiguous k/v [B, S, Hkv, D] into a paged cache -> (k_cache, v_cache, bt)."""
    B, S, Hkv, D = k.shape
    max_blocks = (S + block_size - 1) // block_size
    num_blocks = B * max_blocks
    perm = torch.randperm(num_blocks, generator=generator).to(k.device)
    block_table = perm.reshape(B, max_blocks).to(torch.int32)
    lens = [int(x) for x in seq_lens.tolist()]

    def fill(x: torch.Tensor) -> torch.Tensor:
        cache = 100 * torch.randn(num_blocks, block_size, Hkv, D, generator=generator)
        cache = cache.to(device=x.device, dtype=x.dtype)
        for b in range(B):
            n = lens[b]
            for i in range((n + block_size - 1) // block_size):
                lo, hi = i * block_size, min((i + 1) * block_size, n)
                cache[int(block_table[b, i])][: hi - lo] = x[b, lo:hi]
        return cache

    return fill(k), fill(v), block_table


def ragged_lengths(batch: int, ctx: int, seed: int, lo_frac: float = 0.75) -> list:
    """seq_len ~ U[lo_frac * ctx, ctx] per sequence (seeded, host-side)."""
    g = torch.Generator().manual_seed(seed)
    lo = int(lo_frac * ctx)
    return [int(x) for x in torch.randint(lo, ctx + 1, (batch,), generator=g).tolist()]


def random_paged_workload(lens: Sequence[int], q_heads: int, kv_heads: int, head_dim: int,
                          block_size: int, device, seed: int = 0, spare_blocks: int = 0,
                          dtype=torch.float16, copies: int = 1):
    """Synthetic decode inputs generated on ``device``.

    Returns dict(q, k_cache, v_cache, block_table, seq_lens). Physical blocks are a seeded
    random permutation; block_table rows are zero-padded past each sequence's pages.
    ``copies`` > 1 allocates that many independent caches (list values) so a benchmark can
    rotate through a working set larger than L2.
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
    dg = torch.Generator(device=device).manual_seed(seed + 1)
    q = torch.randn(B, q_heads, head_dim, generator=dg, device=device, dtype=torch.float32)
    shape = (num_blocks, block_size, kv_heads, head_dim)
    ks, vs = [], []
    for _ in range(copies):
        ks.append(torch.randn(shape, generator=dg, device=device, dtype=dtype))
        vs.append(torch.randn(shape, generator=dg, device=device, dtype=dtype))
    return dict(q=q.to(dtype), k_cache=ks[0] if copies == 1 else ks,
                v_cache=vs[0] if copies == 1 else vs, block_table=bt.to(device),
                seq_lens=torch.tensor(list(lens), dtype=torch.int32, device=device),
                num_blocks=num_blocks)
