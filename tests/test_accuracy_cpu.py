"""Synthetic accuracy of the KIVI formats on the CPU (numpy oracle, float64 attention).

No model weights: a needle key planted in a BASELINE-distribution haystack (K ~ N(0, 1) with 4
seeded x10 outlier key channels per kv head, V ~ N(0, 1)), block_size 64. These tests pin the
metric itself and the accuracy each format delivers (oracle/accuracy.py); the GPU tests measure
the same quantities through the decode kernels and compare them with this float64 arithmetic.

Bounds are about twice what two seeds measured, and state each format's accuracy:
  INT8: needle weight within 1% (median over q heads), output rel-RMS mean < 2%;
  FP8:  needle within 3%, output < 8%;  INT4: needle within 10%, output < 30%.
"""
import numpy as np
import pytest

from oracle import accuracy as acc

BOUNDS = {"int8": (1e-2, 2e-2, 5e-2), "fp8": (3e-2, 8e-2, 0.25), "int4": (0.1, 0.3, 0.6)}


@pytest.fixture(scope="module")
def results():
    return {(seed, fmt): acc.format_accuracy(seed, 4096, fmt)
            for seed in (3, 11) for fmt in ("int8", "fp8", "int4")}


def test_needle_takes_about_half_the_mass():
    q, k, v, pos = acc.needle_case(3, 4096)
    _, w = acc.attention64(q, k, v, pos)
    assert 0.3 < float(np.median(w)) < 0.7
    assert (w > 1e-3).all() and (w < 1.0).all()
    # the needle sits in the haystack's middle and only its row was changed
    assert 4096 // 8 <= pos < 4096 - 4096 // 8


def test_attention64_weights_match_the_output():
    """Changing only the needle's value moves the output by exactly w * dv."""
    q, k, v, pos = acc.needle_case(5, 2048)
    o1, w = acc.attention64(q, k, v, pos)
    v2 = v.copy()
    v2[pos] = -v[pos]
    o2, _ = acc.attention64(q, k, v2, pos)
    dv = (v[pos].astype(np.float64) - v2[pos].astype(np.float64))
    group = q.shape[0] // k.shape[1]
    for hq in range(q.shape[0]):
        assert np.allclose(o1[hq] - o2[hq], w[hq] * dv[hq // group], atol=1e-12)


@pytest.mark.parametrize("fmt", ["int8", "fp8", "int4"])
def test_format_accuracy_bounds(results, fmt):
    needle_med, rms_mean, rms_max = BOUNDS[fmt]
    for seed in (3, 11):
        r = results[(seed, fmt)]
        w16, wq = r["needle_weight_fp16"], r["needle_weight"]
        assert float(np.median(np.abs(wq - w16) / w16)) < needle_med
        assert r["out_rel_rms_mean"] < rms_mean
        assert r["out_rel_rms"] < rms_max


def test_formats_rank_by_bits(results):
    for seed in (3, 11):
        e = [results[(seed, f)]["out_rel_rms_mean"] for f in ("int8", "fp8", "int4")]
        assert e[0] < e[1] < e[2]
