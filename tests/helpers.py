"""Shared test helpers: golden fixtures, case builders, the tolerance check."""
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN_DIR = os.path.join(HERE, "golden")

# BASELINE tolerance on fp16 outputs; rel is computed as the reference does
# (tests/test_triton_fp16.py:39: diff / ref.abs().clamp_min(1e-3)).
ATOL = 2e-3
RTOL = 1e-2


def golden_meta():
    with open(os.path.join(GOLDEN_DIR, "golden.json")) as f:
        return json.load(f)["cases"]


_GOLDEN = None


def golden_arrays():
    global _GOLDEN
    if _GOLDEN is None:
        _GOLDEN = dict(np.load(os.path.join(GOLDEN_DIR, "golden.npz")))
    return _GOLDEN


def golden_case(name):
    for c in golden_meta():
        if c["name"] == name:
            return c
    raise KeyError(name)


def errors(out, ref):
    out = np.asarray(out, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    d = np.abs(out - ref)
    if d.size == 0:
        return 0.0, 0.0
    return float(d.max()), float((d / np.maximum(np.abs(ref), 1e-3)).max())


def assert_close(out, ref, atol=ATOL, rtol=RTOL, what=""):
    out = np.asarray(out, dtype=np.float32)
    assert np.isfinite(out).all(), f"{what}: non-finite output"
    max_abs, max_rel = errors(out, ref)
    assert max_abs < atol and max_rel < rtol, \
        f"{what}: max_abs={max_abs:.3e} (tol {atol}) max_rel={max_rel:.3e} (tol {rtol})"
    return max_abs, max_rel


def build_fp16(spec):
    from oracle import cache as oc
    return oc.fp16_case(spec["seed"], spec["lens"], spec["Hq"], spec["Hkv"], spec["D"],
                        spec["block_size"], spec["mode"], spec.get("spare", 64))


def build_quant(spec, garbage=True):
    from oracle import kivi
    return kivi.quant_case(spec["seed"], spec["lens"], spec["Hq"], spec["Hkv"], spec["D"],
                           spec["block_size"], spec["fmt"], spec["mode"], spec.get("spare", 8),
                           garbage=garbage)


def quant_digest(c):
    from oracle import cache as oc
    arrs = [c["q"], c["block_table"], c["seq_lens"]] + [c["cache"][k] for k in sorted(c["cache"])]
    return oc.digest(*arrs)


# ----------------------------------------------------------------------------- torch (GPU) checks

def torch_reference(q, k_cache, v_cache, block_table, seq_lens, scale=None, seqs=None):
    """fp32 torch restatement of the reference oracle (src/bpt/reference.py:20-49), for cases
    too large for the numpy oracle: per sequence, gather its pages, fp32 softmax attention of
    each q head over its kv head (q head h reads kv head h // group). Caches may be fp16 or a
    dequantized fp32 cache. ``seqs`` restricts the work to those sequences (rows of the result
    for other sequences are left NaN). Returns fp32 [B, Hq, D]."""
    import torch
    B, Hq, D = q.shape
    _, bs, Hkv, _ = k_cache.shape
    group = Hq // Hkv
    scale = scale or D ** -0.5
    out = torch.full((B, Hq, D), float("nan"), dtype=torch.float32, device=q.device)
    for b in (range(B) if seqs is None else seqs):
        n = int(seq_lens[b])
        blocks = block_table[b, :(n + bs - 1) // bs].long()
        k = k_cache[blocks].reshape(-1, Hkv, D)[:n].float()
        v = v_cache[blocks].reshape(-1, Hkv, D)[:n].float()
        if n == 0:
            out[b] = 0.0
            continue
        s = torch.einsum("hgd,nhd->hgn", q[b].float().reshape(Hkv, group, D), k) * scale
        out[b] = torch.einsum("hgn,nhd->hgd", torch.softmax(s, dim=-1), v).reshape(Hq, D)
    return out


def torch_dequant_pages(cache, pages):
    """fp32 (k, v) pages [P, bs, H, D] of a bpt KiviCache: x = code * scale + zero, FP8
    e4m3 * scale (the oracle.kivi.dequantize_cache formula, on the GPU)."""
    import torch
    kc, vc = cache.k_codes[pages], cache.v_codes[pages]
    if cache.fmt == "int4":   # keys: low nibble = even channel; values: low nibble = even token
        kc = torch.stack([kc & 0xF, kc >> 4], dim=-1).reshape(*kc.shape[:3], -1)
        vc = torch.stack([vc & 0xF, vc >> 4], dim=2).reshape(vc.shape[0], -1, *vc.shape[2:])
    ks = cache.k_scale[pages].float()[:, None]
    vs = cache.v_scale[pages].float()[..., None]
    if cache.fmt == "fp8":
        return (kc.view(torch.float8_e4m3fn).float() * ks,
                vc.view(torch.float8_e4m3fn).float() * vs)
    return (kc.float() * ks + cache.k_zero[pages].float()[:, None],
            vc.float() * vs + cache.v_zero[pages].float()[..., None])


def torch_reference_kivi(q, cache, block_table, seq_lens, seqs):
    """fp32 reference on the identically dequantized KIVI cache, for the sequences ``seqs``
    (only their pages are dequantized). Returns fp32 [len(seqs), Hq, D]."""
    import torch
    rows = []
    bs = cache.block_size
    for b in seqs:
        n = int(seq_lens[b])
        pages = block_table[b, :(n + bs - 1) // bs].long()
        kd, vd = torch_dequant_pages(cache, pages)
        local = torch.arange(kd.shape[0], dtype=torch.int32, device=q.device)[None]
        rows.append(torch_reference(q[b:b + 1], kd, vd, local, seq_lens[b:b + 1])[0])
    return torch.stack(rows)


def sample_seqs(batch, k, seed=0):
    """k distinct sequence indices (seeded), always including the first and the last."""
    import random
    if batch <= k:
        return list(range(batch))
    rest = random.Random(seed).sample(range(1, batch - 1), k - 2)
    return sorted([0, batch - 1] + rest)
