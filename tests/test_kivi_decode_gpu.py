"""Fused-dequant KIVI decode (INT8 / FP8-E4M3 / INT4) against the reference oracle.

The expected result is the reference's fp32 attention on the identically dequantized cache:
golden outputs made by running src/bpt/reference.py on oracle.kivi.dequantize_cache, and the
numpy oracle on the same cache, at the BASELINE tolerance (max abs 2e-3, max rel 1e-2 with the
reference's clamp_min(1e-3)). Caches carry random garbage in every unused page and in the
unused slots of partial pages, so block-table or masking mistakes cannot pass.
"""
import functools

import numpy as np
import pytest
import torch

from helpers import assert_close, build_quant, golden_arrays, golden_meta
from oracle import attention as oa
from oracle import kivi

pytestmark = pytest.mark.gpu

QUANT_CASES = [c for c in golden_meta() if c["kind"] == "quant"]
SPLITS = [1, 2, 3, 7, None]


def to_gpu_cache(np_cache, fmt, bs):
    from bpt.quant import KiviCache
    t = {k: torch.from_numpy(v.copy()).cuda() for k, v in np_cache.items()}
    return KiviCache(fmt=fmt, block_size=bs, **t)


@functools.lru_cache(maxsize=None)
def _golden_case(name):
    spec = next(c for c in QUANT_CASES if c["name"] == name)
    c = build_quant(spec)
    kd, vd = kivi.dequantize_cache(c["cache"], spec["fmt"])
    ref = oa.paged_decode_attention_ref(c["q"], kd, vd, c["block_table"], c["seq_lens"],
                                        out_dtype=np.float16)
    return spec, c, ref


def _run(c, fmt, bs, num_splits=None):
    from bpt.quant import paged_decode_attention_kivi
    cache = to_gpu_cache(c["cache"], fmt, bs)
    out = paged_decode_attention_kivi(torch.from_numpy(c["q"]).cuda(), cache,
                                      torch.from_numpy(c["block_table"]).cuda(),
                                      torch.from_numpy(c["seq_lens"]).cuda(),
                                      num_splits=num_splits)
    return out.float().cpu().numpy()


@pytest.mark.parametrize("num_splits", SPLITS)
@pytest.mark.parametrize("name", [c["name"] for c in QUANT_CASES])
def test_matches_reference_on_dequantized_cache(name, num_splits):
    spec, c, ref = _golden_case(name)
    out = _run(c, spec["fmt"], spec["block_size"], num_splits)
    assert_close(out, golden_arrays()[name + "/out"], what=f"{name} vs reference")
    assert_close(out, ref, what=f"{name} vs oracle")


@pytest.mark.parametrize("fmt", ["int8", "fp8", "int4"])
@pytest.mark.parametrize("Hq,Hkv,bs,lens", [
    (16, 2, 64, [500, 1, 64]),       # group 8
    (8, 8, 64, [130, 65]),           # MHA
    (16, 8, 16, [300, 17, 16]),      # group 2, 16-token pages
    (32, 8, 32, [257, 31]),          # 32-token pages
    (32, 8, 128, [700, 129, 128]),   # pages larger than a chunk
    (32, 8, 64, [4096, 0, 1, 64, 2000, 4095]),   # very ragged: balanced one-wave splits
])
def test_shapes_and_page_sizes(fmt, Hq, Hkv, bs, lens):
    c = kivi.quant_case(7 + bs + Hq, lens, Hq, Hkv, 128, bs, fmt, "spare", 3)
    kd, vd = kivi.dequantize_cache(c["cache"], fmt)
    ref = oa.paged_decode_attention_ref(c["q"], kd, vd, c["block_table"], c["seq_lens"],
                                        out_dtype=np.float16)
    for ns in (1, 5, None):
        assert_close(_run(c, fmt, bs, ns), ref, what=f"{fmt} Hq={Hq} Hkv={Hkv} bs={bs} ns={ns}")


def test_fp8_nan_codes_in_unused_slots_are_never_read():
    c = kivi.quant_case(11, [70, 33], 32, 8, 128, 64, "fp8", "spare", 2, garbage=True)
    kd, vd = kivi.dequantize_cache(c["cache"], "fp8")
    ref = oa.paged_decode_attention_ref(c["q"], kd, vd, c["block_table"], c["seq_lens"],
                                        out_dtype=np.float16)
    bt = c["block_table"]
    for b, n in enumerate([70, 33]):
        phys = bt[b, (n - 1) // 64]
        c["cache"]["k_codes"][phys, n % 64:] = 0x7F     # e4m3 NaN
        c["cache"]["v_codes"][phys, n % 64:] = 0xFF
    for ns in (1, 3):
        assert_close(_run(c, "fp8", 64, ns), ref, what=f"fp8 NaN garbage ns={ns}")


@pytest.mark.parametrize("fmt", ["int8", "int4"])
def test_partial_states_merge(fmt):
    from bpt.decode import merge_partials
    from bpt.quant import paged_decode_attention_kivi_partial
    spec, c, ref = _golden_case(f"{fmt}_long")
    cache = to_gpu_cache(c["cache"], fmt, spec["block_size"])
    o_part, lse = paged_decode_attention_kivi_partial(
        torch.from_numpy(c["q"]).cuda(), cache, torch.from_numpy(c["block_table"]).cuda(),
        torch.from_numpy(c["seq_lens"]).cuda(), num_splits=6)
    out = merge_partials(o_part, lse).float().cpu().numpy()
    assert_close(out, ref, what="partial + merge")


def torch_dequant(cache, fmt):
    """fp32 dequantization on the GPU (the oracle.kivi.dequantize_cache formula)."""
    kc, vc = cache.k_codes, cache.v_codes
    if fmt == "int4":
        k = torch.stack([kc & 0xF, kc >> 4], dim=-1).reshape(*kc.shape[:3], -1)
        v = torch.stack([vc & 0xF, vc >> 4], dim=2).reshape(vc.shape[0], -1, *vc.shape[2:])
    else:
        k, v = kc, vc
    if fmt == "fp8":
        kf = k.view(torch.float8_e4m3fn).float()
        vf = v.view(torch.float8_e4m3fn).float()
        return kf * cache.k_scale.float()[:, None], vf * cache.v_scale.float()[..., None]
    kf = k.float() * cache.k_scale.float()[:, None] + cache.k_zero.float()[:, None]
    vf = v.float() * cache.v_scale.float()[..., None] + cache.v_zero.float()[..., None]
    return kf, vf


@pytest.mark.parametrize("fmt,B", [("int8", 8), ("fp8", 8), ("int4", 8), ("int8", 32),
                                   ("fp8", 32), ("int4", 64)])
def test_full_size_quantized_batch(fmt, B):
    """B x ctx 32k at the BASELINE KIVI configurations (INT8 / FP8 B=32, INT4 B=64, and B=8),
    quantized on the GPU by the append kernel, decoded, and checked against torch fp32
    attention on the dequantized cache."""
    from bpt.cache import ragged_lengths
    from bpt.quant import empty_kivi_cache, paged_decode_attention_kivi, quantize_append
    from helpers import torch_reference
    ctx, bs, Hq, Hkv, D = 32768, 64, 32, 8, 128
    lens = ragged_lengths(B, ctx, seed=3)
    g = torch.Generator(device="cuda").manual_seed(5)
    k = torch.randn(B, ctx, Hkv, D, device="cuda", generator=g, dtype=torch.float16)
    v = torch.randn(B, ctx, Hkv, D, device="cuda", generator=g, dtype=torch.float16)
    q = torch.randn(B, Hq, D, device="cuda", generator=g, dtype=torch.float16)
    pages = ctx // bs
    bt = torch.randperm(B * pages, device="cuda").reshape(B, pages).to(torch.int32)
    cache = empty_kivi_cache(B * pages, bs, Hkv, D, fmt)
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    quantize_append(cache, k, v, sl, torch.zeros_like(sl), bt)
    kd, vd = torch_dequant(cache, fmt)
    ref = torch_reference(q, kd, vd, bt, sl)
    del k, v
    for ns in (None, 1):
        out = paged_decode_attention_kivi(q, cache, bt, sl, num_splits=ns)
        assert_close(out.float().cpu().numpy(), ref.cpu().numpy(), what=f"{fmt} B={B} ctx=32k")


@pytest.mark.parametrize("fmt", ["int8", "fp8", "int4"])
def test_decode_with_fp16_residual(fmt):
    """A decode loop's view of a KIVI cache: full pages quantized, the newest tokens (a
    partial page, 0..63 of them) still fp16. paged_decode_attention_kivi_with_residual must
    equal fp32 attention over [dequantized pages ; fp16 residual] (numpy, per sequence)."""
    from bpt.quant import paged_decode_attention_kivi_with_residual
    from oracle.cache import block_table_for, make_qkv, rng
    bs, Hq, Hkv, D, R = 64, 32, 8, 128, 64
    total = [300, 64, 5, 1000, 127]
    nq = [(n // bs) * bs for n in total]            # quantized, page-aligned
    nr = [n - m for n, m in zip(total, nq)]         # residual, < one page
    g = rng(21)
    q, k, v = make_qkv(g, total, Hq, Hkv, D, outlier_channels=4)
    bt, nb = block_table_for(g, [max(m, 1) for m in nq], bs, "spare", 4)
    cache = kivi.empty_cache(nb, bs, Hkv, D, fmt)
    kivi.quantize_append(cache, k, v, nq, [0] * len(total), bt, bs, fmt)
    kd, vd = kivi.dequantize_cache(cache, fmt)
    k_res = np.zeros((len(total), R, Hkv, D), np.float16)
    v_res = np.zeros_like(k_res)
    for b, (m, r) in enumerate(zip(nq, nr)):
        k_res[b, :r] = k[b, m:m + r]
        v_res[b, :r] = v[b, m:m + r]
    # reference: fp32 attention over the dequantized pages followed by the fp16 residual
    ref = np.zeros((len(total), Hq, D), np.float32)
    group = Hq // Hkv
    for b, (m, r) in enumerate(zip(nq, nr)):
        pages = bt[b, :(m + bs - 1) // bs]
        kk = np.concatenate([kd[pages].reshape(-1, Hkv, D)[:m], k_res[b, :r].astype(np.float32)])
        vv = np.concatenate([vd[pages].reshape(-1, Hkv, D)[:m], v_res[b, :r].astype(np.float32)])
        for hq in range(Hq):
            s = kk[:, hq // group] @ q[b, hq].astype(np.float32) / np.sqrt(D)
            p = np.exp(s - s.max())
            ref[b, hq] = (p / p.sum()) @ vv[:, hq // group]
    gc = to_gpu_cache(cache, fmt, bs)
    args = (torch.from_numpy(q).cuda(), gc, torch.from_numpy(bt).cuda(),
            torch.tensor(nq, dtype=torch.int32, device="cuda"),
            torch.from_numpy(k_res).cuda(), torch.from_numpy(v_res).cuda(),
            torch.tensor(nr, dtype=torch.int32, device="cuda"))
    for ns in (None, 1):
        out = paged_decode_attention_kivi_with_residual(*args, num_splits=ns)
        assert_close(out.float().cpu().numpy(), ref, what=f"{fmt} residual ns={ns}")


@pytest.mark.parametrize("fmt,B", [("int4", 64), ("int4", 32), ("int8", 32)])
def test_full_size_decode_is_deterministic(fmt, B):
    """Repeated calls give bitwise-identical outputs at several split counts. The compute warps
    share per-page q scale entries in shared memory; a warp that raced ahead into the next
    chunk must not overwrite the entries another warp is still reading (an earlier version did,
    rarely, at some split counts)."""
    from bpt.cache import ragged_lengths
    from bpt.quant import empty_kivi_cache, paged_decode_attention_kivi, quantize_append
    ctx, bs, Hq, Hkv, D = 32768, 64, 32, 8, 128
    lens = ragged_lengths(B, ctx, seed=3)
    g = torch.Generator(device="cuda").manual_seed(5)
    k = torch.randn(B, ctx, Hkv, D, device="cuda", generator=g, dtype=torch.float16)
    v = torch.randn(B, ctx, Hkv, D, device="cuda", generator=g, dtype=torch.float16)
    q = torch.randn(B, Hq, D, device="cuda", generator=g, dtype=torch.float16)
    pages = ctx // bs
    bt = torch.randperm(B * pages, device="cuda").reshape(B, pages).to(torch.int32)
    cache = empty_kivi_cache(B * pages, bs, Hkv, D, fmt)
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    quantize_append(cache, k, v, sl, torch.zeros_like(sl), bt)
    del k, v
    for ns in (None, 1, 5, 7):
        first = paged_decode_attention_kivi(q, cache, bt, sl, num_splits=ns)
        for _ in range(4):
            assert torch.equal(first, paged_decode_attention_kivi(q, cache, bt, sl, num_splits=ns)), \
                f"{fmt} B={B} num_splits={ns}: outputs differ between calls"
