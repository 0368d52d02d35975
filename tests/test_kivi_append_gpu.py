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
