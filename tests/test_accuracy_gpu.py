"""Synthetic accuracy of the KIVI formats through the decode kernels (GPU).

bpt.accuracy.needle_study measures, through bpt's fp16 and KIVI kernels, the needle's
attention weight per q head (two decodes whose caches differ only in the needle's value) and
the output error of a format against the fp16 cache. Checked here against float64 attention on
the same tensors (the fp16 cache, and the cache dequantized from the codes the append kernel
wrote), at 4k, 32k and 128k tokens, and against the numpy oracle on identical inputs at 4k.
The format bounds are the ones tests/test_accuracy_cpu.py states.
"""
import math

import numpy as np
import pytest
import torch

from helpers import torch_dequant_pages

pytestmark = pytest.mark.gpu

BOUNDS = {"int8": (1e-2, 2e-2, 5e-2), "fp8": (3e-2, 8e-2, 0.25), "int4": (0.1, 0.3, 0.6)}


def attention64(q, k, v, pos):
    """float64 attention of q [Hq, D] over k, v [n, Hkv, D]: (out [Hq, D], needle weight)."""
    Hq, D = q.shape
    Hkv = k.shape[1]
    qf = q.double().reshape(Hkv, Hq // Hkv, D)
    s = torch.einsum("hgd,nhd->hgn", qf, k.double()) / math.sqrt(D)
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hgn,nhd->hgd", p, v.double()).reshape(Hq, D), p[..., pos].reshape(Hq)


def dequantized(fmt, k, v, block_size=64):
    from bpt.quant import empty_kivi_cache, quantize_append
    n, H, D = k.shape
    pages = (n + block_size - 1) // block_size
    bt = torch.arange(pages, dtype=torch.int32, device=k.device)[None]
    sl = torch.tensor([n], dtype=torch.int32, device=k.device)
    cache = empty_kivi_cache(pages, block_size, H, D, fmt, device=k.device)
    quantize_append(cache, k[None], v[None], sl, torch.zeros_like(sl), bt)
    kd, vd = torch_dequant_pages(cache, torch.arange(pages, device=k.device))
    return kd.reshape(-1, H, D)[:n], vd.reshape(-1, H, D)[:n]


@pytest.mark.parametrize("ctx", [4096, 32768, 131072])
@pytest.mark.parametrize("fmt", ["int8", "fp8", "int4"])
def test_needle_study_through_the_kernels(fmt, ctx):
    from bpt.accuracy import needle_inputs, needle_study
    inputs = needle_inputs(ctx, seed=5 + ctx % 7, device="cuda")
    r = needle_study(fmt, ctx, inputs=inputs)
    q, k, v, pos = inputs
    o16, w16 = attention64(q, k, v, pos)
    kd, vd = dequantized(fmt, k, v)
    oq, wq = attention64(q, kd, vd, pos)
    # the kernel-measured weights are the float64 weights (fp16 outputs limit the agreement)
    assert (r["needle_weight_fp16"].double() - w16.cpu()).abs().max() < 2e-3
    assert (r["needle_weight"].double() - wq.cpu()).abs().max() < 2e-3
    # the decoded outputs themselves are within the BASELINE tolerance of float64
    for got, ref in ((r["outputs"]["fp16"], o16), (r["outputs"][fmt], oq)):
        d = (got.double() - ref.cpu()).abs()
        assert d.max() < 2e-3 and (d / ref.cpu().abs().clamp_min(1e-3)).max() < 1e-2
    # the study's output error is the format's: it matches float64 to 10%
    rel64 = ((oq - o16).norm(dim=-1) / o16.norm(dim=-1)).cpu()
    assert abs(r["out_rel_rms_mean"] - float(rel64.mean())) < 0.1 * float(rel64.mean()) + 1e-4
    needle_med, rms_mean, rms_max = BOUNDS[fmt]
    assert r["needle_rel_err_median"] < needle_med
    assert r["out_rel_rms_mean"] < rms_mean and r["out_rel_rms"] < rms_max


def test_needle_study_matches_the_numpy_oracle():
    """Identical inputs (numpy-generated, uploaded): the kernels' needle weights and format
    error agree with oracle.accuracy's float64 figures."""
    from bpt.accuracy import needle_study
    from oracle import accuracy as acc
    q, k, v, pos = acc.needle_case(3, 4096)
    dev = [torch.from_numpy(x).cuda() for x in (q, k, v)]
    for fmt in ("int8", "fp8", "int4"):
        r = needle_study(fmt, 4096, inputs=(*dev, pos))
        ref = acc.format_accuracy(3, 4096, fmt)
        assert np.abs(r["needle_weight_fp16"].numpy() - ref["needle_weight_fp16"]).max() < 2e-3
        assert np.abs(r["needle_weight"].numpy() - ref["needle_weight"]).max() < 2e-3
        assert abs(r["out_rel_rms_mean"] - ref["out_rel_rms_mean"]) < 0.1 * ref["out_rel_rms_mean"]
