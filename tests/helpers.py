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
