"""Pin the CPU oracle to the reference (CPU-only).

The golden outputs were produced by the reference's own ``paged_decode_attention_ref``
(src/bpt/reference.py:20-49) by tests/golden/make_golden.py. The numpy restatement in
``oracle/`` must reproduce them (fp32 math, so within a few fp16 ulps), and must also pass the
reference's own oracle checks (tests/test_reference.py: agreement with SDPA on a contiguous
cache, invariance to block permutation and garbage).
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from helpers import (build_fp16, build_quant, errors, golden_arrays, golden_meta,
                     quant_digest)
from oracle import attention as oa
from oracle import cache as oc
from oracle import kivi

FP16_CASES = [c for c in golden_meta() if c["kind"] == "fp16"]
QUANT_CASES = [c for c in golden_meta() if c["kind"] == "quant"]
CODE_CASES = [c for c in golden_meta() if c["kind"] == "codes"]

# oracle vs reference: identical math up to fp32 summation order -> a few fp16 ulps
ORACLE_ATOL, ORACLE_RTOL = 1e-3, 2e-3


@pytest.mark.parametrize("spec", FP16_CASES, ids=lambda s: s["name"])
def test_oracle_matches_reference_fp16(spec):
    c = build_fp16(spec)
    assert oc.digest(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                     c["seq_lens"]) == spec["digest"], "input generator drifted"
    out = oa.paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                        c["seq_lens"])
    a, r = errors(out, golden_arrays()[spec["name"] + "/out"])
    assert a < ORACLE_ATOL and r < ORACLE_RTOL, (a, r)


@pytest.mark.parametrize("spec", QUANT_CASES, ids=lambda s: s["name"])
def test_oracle_matches_reference_on_dequantized_cache(spec):
    c = build_quant(spec)
    assert quant_digest(c) == spec["digest"], "quantizer or generator drifted"
    kd, vd = kivi.dequantize_cache(c["cache"], spec["fmt"])
    out = oa.paged_decode_attention_ref(c["q"], kd, vd, c["block_table"], c["seq_lens"],
                                        out_dtype=np.float16)
    a, r = errors(out, golden_arrays()[spec["name"] + "/out"])
    assert a < ORACLE_ATOL and r < ORACLE_RTOL, (a, r)


@pytest.mark.parametrize("spec", CODE_CASES, ids=lambda s: s["name"])
def test_quantizer_matches_golden_codes(spec):
    c = build_quant(spec, garbage=False)
    g = golden_arrays()
    for k, arr in c["cache"].items():
        np.testing.assert_array_equal(arr, g[spec["name"] + "/" + k], err_msg=k)


# ------------------------------------------------------ the reference's own oracle checks

def _sdpa(q, k, v, lens):
    B, Hq, D = q.shape
    group = Hq // k.shape[2]
    outs = []
    for b in range(B):
        n = int(lens[b])
        kb = k[b, :n].repeat_interleave(group, dim=1).permute(1, 0, 2)
        vb = v[b, :n].repeat_interleave(group, dim=1).permute(1, 0, 2)
        outs.append(F.scaled_dot_product_attention(q[b][:, None, :], kb, vb)[:, 0])
    return torch.stack(outs)


@pytest.mark.parametrize("lens", [[1], [37], [100, 33, 1, 64]])
@pytest.mark.parametrize("block_size", [16, 32])
@pytest.mark.parametrize("Hq,Hkv,D", [(32, 8, 128), (4, 4, 64), (8, 1, 64)])
def test_oracle_matches_sdpa(Hq, Hkv, D, block_size, lens):
    """Restates tests/test_reference.py:36-58 for the numpy oracle (fp32 inputs, atol 1e-5)."""
    g = oc.rng(3)
    B = len(lens)
    q = g.standard_normal((B, Hq, D), dtype=np.float32)
    k = g.standard_normal((B, max(lens), Hkv, D), dtype=np.float32)
    v = g.standard_normal((B, max(lens), Hkv, D), dtype=np.float32)
    kc, vc, bt, _ = oc.build_paged_cache(k, v, lens, block_size, g)
    out = oa.paged_decode_attention_ref(q, kc, vc, bt, np.asarray(lens))
    ref = _sdpa(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v), lens).numpy()
    assert np.abs(out - ref).max() < 1e-5


def test_oracle_ignores_permutation_and_garbage():
    """Restates tests/test_reference.py:61-69."""
    lens = [37, 5]
    g = oc.rng(4)
    q = g.standard_normal((2, 8, 32), dtype=np.float32)
    k = g.standard_normal((2, 37, 2, 32), dtype=np.float32)
    v = g.standard_normal((2, 37, 2, 32), dtype=np.float32)
    a = oc.build_paged_cache(k, v, lens, 16, oc.rng(1))
    b = oc.build_paged_cache(k, v, lens, 16, oc.rng(2))
    out_a = oa.paged_decode_attention_ref(q, a[0], a[1], a[2], np.asarray(lens))
    out_b = oa.paged_decode_attention_ref(q, b[0], b[1], b[2], np.asarray(lens))
    assert np.allclose(out_a, out_b, atol=1e-6)


def test_partial_states_merge_to_full():
    """Split states + LSE merge (triton_fp16.py:138-163) equal one pass over the sequence."""
    c = oc.fp16_case(5, [300, 77, 1, 0], 32, 8, 128, 16, "spare", 4)
    full = oa.paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                         c["seq_lens"], out_dtype=np.float32)
    lens = c["seq_lens"]
    cuts = [np.zeros_like(lens), lens // 3, (2 * lens) // 3, lens]
    parts = [oa.paged_decode_attention_partial(c["q"], c["k_cache"], c["v_cache"],
                                               c["block_table"], lens, lo, hi)
             for lo, hi in zip(cuts[:-1], cuts[1:])]
    merged = oa.merge_states([p[0] for p in parts], [p[1] for p in parts])
    assert np.abs(merged - full).max() < 1e-5


def test_empty_sequence_is_zero():
    c = oc.fp16_case(6, [0, 3], 4, 2, 64, 16, "spare", 2)
    out = oa.paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                        c["seq_lens"])
    assert np.all(out[0] == 0)
