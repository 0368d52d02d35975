"""bpt against the reference's own Triton FP16 kernel, on the same B200 and the same inputs.

The reference package is installed offline under baseline/_ref (git-ignored); its
src/bpt/triton_fp16.py is loaded by path (the installed package is also named `bpt`). These
tests skip when it is absent. They run every golden FP16 case (the reference's test shapes,
block sizes and ragged lengths) plus full-size BASELINE shapes through both kernels, for the
reference's heuristic split and forced split counts, and hold the two outputs to the
criterion the reference holds its own kernel to against its oracle: max abs < 2e-3
(tests/test_triton_fp16.py:25-42). A relative bound does not apply between the two kernels:
the reference rounds P to fp16 before P.V (src/bpt/triton_fp16.py:135), which costs up to
~5 % relative on outputs near zero, while bpt keeps P at ~22 bits. On the golden cases bpt must
also be at least as close to the reference's fp32 oracle output as the Triton kernel is.
"""
import functools
import importlib.util
import os

import numpy as np
import pytest
import torch

from helpers import ATOL, build_fp16, golden_arrays, golden_meta

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_PATH = os.path.join(ROOT, "baseline", "_ref", "bpt", "triton_fp16.py")


@functools.lru_cache(maxsize=None)
def _ref():
    if not os.path.exists(REF_PATH):
        pytest.skip("reference not installed under baseline/_ref")
    spec = importlib.util.spec_from_file_location("bpt_reference_triton_fp16", REF_PATH)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


# the reference asserts seq_lens >= 1 (triton_fp16.py:201): cases with empty sequences are
# compared by the oracle tests only
FP16_CASES = [c for c in golden_meta() if c["kind"] == "fp16" and min(c["lens"]) >= 1]


def _gpu(c):
    return (torch.from_numpy(c["q"]).cuda(), torch.from_numpy(c["k_cache"]).cuda(),
            torch.from_numpy(c["v_cache"]).cuda(), torch.from_numpy(c["block_table"]).cuda(),
            torch.from_numpy(c["seq_lens"]).cuda())


@pytest.mark.parametrize("num_splits", [None, 1, 4])
@pytest.mark.parametrize("name", [c["name"] for c in FP16_CASES])
def test_matches_reference_triton_on_golden_cases(name, num_splits):
    from bpt import paged_decode_attention
    ref = _ref()
    spec = next(c for c in FP16_CASES if c["name"] == name)
    args = _gpu(build_fp16(spec))
    tri = ref.paged_decode_attention_triton(*args, num_splits=num_splits).float().cpu().numpy()
    got = paged_decode_attention(*args, num_splits=num_splits).float().cpu().numpy()
    assert np.isfinite(got).all()
    d = float(np.abs(got - tri).max())
    assert d < ATOL, f"{name} splits={num_splits}: max abs vs reference Triton {d:.3e}"
    gold = golden_arrays()[name + "/out"].astype(np.float32)
    e_bpt = float(np.abs(got - gold).max())
    e_tri = float(np.abs(tri - gold).max())
    assert e_bpt <= max(e_tri, 2.0 ** -11), (name, num_splits, e_bpt, e_tri)


@pytest.mark.parametrize("batch,ctx,ragged", [(8, 16384, True), (1, 65536, False),
                                              (32, 4096, True)])
def test_matches_reference_triton_at_baseline_shapes(batch, ctx, ragged):
    from bpt import paged_decode_attention
    from bpt.cache import ragged_lengths, random_paged_workload
    ref = _ref()
    lens = ragged_lengths(batch, ctx, 1234) if ragged else [ctx] * batch
    w = random_paged_workload(lens, 32, 8, 128, 16, "cuda", seed=7)
    args = (w["q"], w["k_cache"], w["v_cache"], w["block_table"], w["seq_lens"])
    want = ref.paged_decode_attention_triton(*args).float()
    got = paged_decode_attention(*args).float()
    d = (got - want).abs().max().item()
    assert d < ATOL, f"B={batch} ctx={ctx}: max abs vs reference Triton {d:.3e}"
