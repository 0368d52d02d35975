"""The CUDA cache-append quantizer is bit-exact with the numpy KIVI specification.

Every array of the cache (codes, fp16 scales, fp16 zero-points) must match oracle/kivi.py
byte for byte: INT8, FP8-E4M3 and INT4, several page sizes, ragged lengths with partial last
pages, appends in two steps at a page-aligned offset, and adversarial values (constant
channels -> scale 0, subnormal scales, values near the fp16 maximum, signed zeros, ties).
"""
import numpy as np
import pytest
import torch

from oracle import cache as oc
from oracle import kivi

pytestmark = pytest.mark.gpu

FORMATS = ["int8", "fp8", "int4"]


def _gpu_cache(np_cache, fmt, bs):
    from bpt.quant import KiviCache
    t = {k: torch.from_numpy(v.copy()).cuda() for k, v in np_cache.items()}
    return KiviCache(fmt=fmt, block_size=bs, **t)


def _compare(gpu_cache, np_cache):
    for name, ref in np_cache.items():
        got = getattr(gpu_cache, name).cpu().numpy()
        if ref.dtype == np.float16:
            np.testing.assert_array_equal(got.view(np.uint16), ref.view(np.uint16), err_msg=name)
        else:
            np.testing.assert_array_equal(got, ref, err_msg=name)


def _append_both(np_cache, gcache, k, v, lens, start, bt, bs, fmt):
    from bpt.quant import quantize_append
    kivi.quantize_append(np_cache, k, v, lens, start, bt, bs, fmt)
    quantize_append(gcache, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(),
                    torch.tensor(lens, dtype=torch.int32, device="cuda"),
                    torch.tensor(start, dtype=torch.int32, device="cuda"),
                    torch.from_numpy(bt).cuda())
    torch.cuda.synchronize()


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("bs", [16, 64, 128])
def test_append_bit_exact(fmt, bs):
    lens = [1, bs - 1, bs, bs + 1, 3 * bs + 5]
    g = oc.rng(50 + bs)
    _, k, v = oc.make_qkv(g, lens, 4, 8, 128, outlier_channels=4)
    bt, nb = oc.block_table_for(g, lens, bs, "spare", 3)
    ref = kivi.empty_cache(nb, bs, 8, 128, fmt)
    gc = _gpu_cache(kivi.empty_cache(nb, bs, 8, 128, fmt), fmt, bs)
    _append_both(ref, gc, k, v, lens, [0] * len(lens), bt, bs, fmt)
    _compare(gc, ref)


@pytest.mark.parametrize("fmt", FORMATS)
def test_append_in_two_steps(fmt):
    bs = 64
    lens_total = [300, 64, 129]
    g = oc.rng(60)
    _, k, v = oc.make_qkv(g, lens_total, 4, 8, 128, outlier_channels=4)
    bt, nb = oc.block_table_for(g, lens_total, bs, "spare", 2)
    first = [128, 64, 64]
    second = [n - f for n, f in zip(lens_total, first)]
    ref = kivi.empty_cache(nb, bs, 8, 128, fmt)
    gc = _gpu_cache(kivi.empty_cache(nb, bs, 8, 128, fmt), fmt, bs)
    _append_both(ref, gc, k[:, :max(first)].copy(), v[:, :max(first)].copy(), first,
                 [0, 0, 0], bt, bs, fmt)
    k2 = np.zeros_like(k)
    v2 = np.zeros_like(v)
    for b, f in enumerate(first):
        k2[b, :lens_total[b] - f] = k[b, f:lens_total[b]]
        v2[b, :lens_total[b] - f] = v[b, f:lens_total[b]]
    _append_both(ref, gc, k2, v2, second, first, bt, bs, fmt)
    _compare(gc, ref)


@pytest.mark.parametrize("fmt", FORMATS)
def test_append_adversarial_values(fmt):
    bs, H, D = 16, 2, 128
    lens = [16, 9]
    g = oc.rng(70)
    x = g.standard_normal((2, 16, H, D), dtype=np.float32)
    x[:, :, 0, 0] = 3.0                                   # constant channel -> scale 0
    x[:, :, 0, 1] = 1e-6 * g.standard_normal((2, 16))     # subnormal-range scale
    x[:, :, 0, 2] = 6e4 * np.sign(g.standard_normal((2, 16)))   # near fp16 max
    x[:, :, 0, 3] = -0.0
    x[:, 3, 1, :] = 0.0                                   # a zero value row
    x[:, 4, 1, :] = np.linspace(-1, 1, D)                 # evenly spaced: rounding ties
    x[:, 5, 1, :] = 448.0 * np.linspace(-1, 1, D)
    k = x.astype(np.float16)
    v = (x[:, :, ::-1] * 0.5).astype(np.float16).copy()
    bt, nb = oc.block_table_for(g, lens, bs, "spare", 1)
    ref = kivi.empty_cache(nb, bs, H, D, fmt)
    gc = _gpu_cache(kivi.empty_cache(nb, bs, H, D, fmt), fmt, bs)
    _append_both(ref, gc, k, v, lens, [0, 0], bt, bs, fmt)
    _compare(gc, ref)


def test_append_matches_golden_codes():
    """The committed golden codes (numpy spec) are reproduced by the CUDA kernel too."""
    from helpers import build_quant, golden_arrays, golden_meta
    for spec in [c for c in golden_meta() if c["kind"] == "codes"]:
        c = build_quant(spec, garbage=False)
        fmt, bs = spec["fmt"], spec["block_size"]
        gc = _gpu_cache(kivi.empty_cache(c["num_blocks"], bs, spec["Hkv"], spec["D"], fmt),
                        fmt, bs)
        from bpt.quant import quantize_append
        quantize_append(gc, torch.from_numpy(c["k"]).cuda(), torch.from_numpy(c["v"]).cuda(),
                        torch.from_numpy(c["seq_lens"]).cuda(),
                        torch.zeros(len(spec["lens"]), dtype=torch.int32, device="cuda"),
                        torch.from_numpy(c["block_table"]).cuda())
        gold = {k: v for k, v in golden_arrays().items() if k.startswith(spec["name"] + "/")}
        _compare(gc, {k.split("/", 1)[1]: v for k, v in gold.items()})


@pytest.mark.parametrize("fmt", FORMATS)
def test_append_error_bound_at_full_size(fmt):
    """Size-independent properties of the GPU quantizer at the BASELINE KIVI size (B=8 x 32k
    tokens, bs=64, 8 kv heads, D=128; N(0,1) keys with x10 outlier channels): every valid
    dequantized value is within the rounding bound of the KIVI formula.
    INT8 / INT4: |x - x_hat| <= s/2 + (Q s + |z|) 2^-10, where s and z are rounded to fp16.
    FP8: |x - x_hat| <= |x| 2^-4 + s 2^-2 (e4m3 round-half-even, clamp at 448 s).
    Codes stay inside the format's range."""
    from bpt.quant import empty_kivi_cache, quantize_append
    from test_kivi_decode_gpu import torch_dequant
    B, ctx, bs, H, D = 8, 32768, 64, 8, 128
    g = torch.Generator(device="cuda").manual_seed(11)
    k = torch.randn(B, ctx, H, D, device="cuda", generator=g, dtype=torch.float16)
    k[:, :, :, :4] *= 10   # outlier channels
    v = torch.randn(B, ctx, H, D, device="cuda", generator=g, dtype=torch.float16)
    lens = torch.randint(ctx // 2, ctx + 1, (B,), device="cuda", generator=g).to(torch.int32)
    pages = ctx // bs
    bt = torch.randperm(B * pages, device="cuda").reshape(B, pages).to(torch.int32)
    cache = empty_kivi_cache(B * pages, bs, H, D, fmt)
    quantize_append(cache, k, v, lens, torch.zeros_like(lens), bt)
    torch.cuda.synchronize()
    kd, vd = torch_dequant(cache, fmt)                   # [nb, bs, H, D] fp32
    # originals in page layout, and which slots hold a valid token
    kp = torch.zeros_like(kd)
    vp = torch.zeros_like(vd)
    valid = torch.zeros(B * pages, bs, dtype=torch.bool, device="cuda")
    tok = torch.arange(ctx, device="cuda")
    for b in range(B):
        kp[bt[b]] = k[b].float().view(pages, bs, H, D)
        vp[bt[b]] = v[b].float().view(pages, bs, H, D)
        valid[bt[b]] = (tok < lens[b]).view(pages, bs)
    m = valid[:, :, None, None]
    ks = cache.k_scale.float()[:, None, :, :]            # per page, head, channel
    vs = cache.v_scale.float()[:, :, :, None]            # per token, head
    if fmt == "fp8":
        kb = kp.abs() * 2.0 ** -4 + ks * 0.25
        vb = vp.abs() * 2.0 ** -4 + vs * 0.25
    else:
        Q = 255.0 if fmt == "int8" else 15.0
        kz = cache.k_zero.float()[:, None, :, :]
        vz = cache.v_zero.float()[:, :, :, None]
        kb = ks * 0.5 + (Q * ks + kz.abs()) * 2.0 ** -10 + 1e-6
        vb = vs * 0.5 + (Q * vs + vz.abs()) * 2.0 ** -10 + 1e-6
        top = int(Q)
        codes_k = cache.k_codes if fmt == "int8" else torch.stack(
            [cache.k_codes & 15, cache.k_codes >> 4], -1)
        codes_v = cache.v_codes if fmt == "int8" else torch.stack(
            [cache.v_codes & 15, cache.v_codes >> 4], -1)
        assert int(codes_k.max()) <= top and int(codes_v.max()) <= top
    assert bool((cache.k_scale.float() >= 0).all()) and bool((cache.v_scale.float() >= 0).all())
    ek = ((kd - kp).abs() - kb).masked_fill(~m, -1.0)
    ev = ((vd - vp).abs() - vb).masked_fill(~m, -1.0)
    assert float(ek.max()) <= 0.0, f"{fmt} keys exceed the bound by {float(ek.max()):.3e}"
    assert float(ev.max()) <= 0.0, f"{fmt} values exceed the bound by {float(ev.max()):.3e}"
