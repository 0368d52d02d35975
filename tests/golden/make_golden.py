"""Generate the golden fixtures from the REFERENCE implementation itself.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py --reference-dir DIR   (or BPT_REFERENCE_DIR=DIR)

It loads ``src/bpt/reference.py`` of the reference by file path (the new package is also
called ``bpt``, so a normal import would collide), builds every case's inputs with the seeded
numpy builders in ``oracle/`` and runs the reference's ``paged_decode_attention_ref`` (torch,
fp32 math, CPU). Inputs are not stored: they are regenerated from the seed on any machine and
checked against the stored digest. What is stored per case is the spec, the input digest and
the reference's fp16 output. For the KIVI cases the reference runs on the fp32 cache produced
by ``oracle.kivi.dequantize_cache`` ("fp32 math on the identically dequantized cache"), and a
small cache's codes/scales are stored verbatim to pin the quantizer specification.

The result is ``tests/golden/golden.npz`` + ``tests/golden/golden.json``.
"""
import argparse
import importlib.util
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import cache as oc  # noqa: E402
from oracle import kivi  # noqa: E402

# (Hq, Hkv, D): Llama-3-8B, MHA, MQA -- the reference's own shape list
# (tests/test_reference.py:9, tests/test_triton_fp16.py:9)
SHAPES = [(32, 8, 128), (4, 4, 64), (8, 1, 64)]
# ragged lengths of tests/test_triton_fp16.py:28
LENS = [[1], [37], [100, 33, 1, 64], [4096, 1000, 17, 2049]]
BLOCK_SIZES = [16, 32]


def fp16_specs():
    specs = []
    seed = 100
    for (Hq, Hkv, D) in SHAPES:
        for bs in BLOCK_SIZES:
            for lens in LENS:
                specs.append(dict(kind="fp16", seed=seed, lens=lens, Hq=Hq, Hkv=Hkv, D=D,
                                  block_size=bs, mode="reference"))
                seed += 1
    # BASELINE CPU-correctness configuration
    specs.append(dict(kind="fp16", seed=0, lens=[4096, 2731], Hq=32, Hkv=8, D=128,
                      block_size=16, mode="spare", spare=64, name="c1"))
    # empty and single-token sequences mixed in one batch, zero-padded table
    specs.append(dict(kind="fp16", seed=7, lens=[0, 5, 16, 17, 0, 1], Hq=32, Hkv=8, D=128,
                      block_size=16, mode="spare", spare=8, name="empty_mix"))
    # block_size 64 and 128 pages (page larger than one 64-token chunk)
    specs.append(dict(kind="fp16", seed=8, lens=[300, 64, 129], Hq=32, Hkv=8, D=128,
                      block_size=64, mode="spare", spare=8, name="bs64"))
    specs.append(dict(kind="fp16", seed=9, lens=[300, 128, 1], Hq=32, Hkv=8, D=128,
                      block_size=128, mode="spare", spare=4, name="bs128"))
    for s in specs:
        s.setdefault("name", "fp16_h{Hq}_{Hkv}_d{D}_bs{block_size}_l{n}".format(
            n="-".join(map(str, s["lens"])), **s))
    return specs


def quant_specs():
    specs = []
    for i, fmt in enumerate(kivi.FORMATS):
        specs.append(dict(kind="quant", fmt=fmt, seed=200 + i, lens=[1, 63, 64, 65, 200, 0],
                          Hq=32, Hkv=8, D=128, block_size=64, mode="spare", spare=8,
                          name=f"{fmt}_mixed"))
        specs.append(dict(kind="quant", fmt=fmt, seed=210 + i, lens=[2000, 777], Hq=32,
                          Hkv=8, D=128, block_size=64, mode="spare", spare=8,
                          name=f"{fmt}_long"))
    return specs


def code_specs():
    """Small caches whose quantized arrays are stored verbatim (quantizer spec pins)."""
    return [dict(kind="codes", fmt=fmt, seed=300 + i, lens=[70, 64, 3], Hq=4, Hkv=2, D=128,
                 block_size=64, mode="spare", spare=2, name=f"codes_{fmt}")
            for i, fmt in enumerate(kivi.FORMATS)]


def build_fp16(spec):
    return oc.fp16_case(spec["seed"], spec["lens"], spec["Hq"], spec["Hkv"], spec["D"],
                        spec["block_size"], spec["mode"], spec.get("spare", 64))


def build_quant(spec, garbage=True):
    return kivi.quant_case(spec["seed"], spec["lens"], spec["Hq"], spec["Hkv"], spec["D"],
                           spec["block_size"], spec["fmt"], spec["mode"], spec.get("spare", 8),
                           garbage=garbage)


def quant_digest(c):
    arrs = [c["q"], c["block_table"], c["seq_lens"]] + [c["cache"][k]
                                                       for k in sorted(c["cache"])]
    return oc.digest(*arrs)


def load_reference(ref_dir):
    path = os.path.join(ref_dir, "src", "bpt", "reference.py")
    spec = importlib.util.spec_from_file_location("bpt_reference_oracle", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def run_reference(ref, q, kc, vc, bt, sl):
    import torch
    with torch.no_grad():
        out = ref.paged_decode_attention_ref(
            torch.from_numpy(q), torch.from_numpy(np.ascontiguousarray(kc)),
            torch.from_numpy(np.ascontiguousarray(vc)), torch.from_numpy(bt),
            torch.from_numpy(sl))
    return out.numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-dir", default=os.environ.get("BPT_REFERENCE_DIR"),
                    help="checkout of the reference project (or set BPT_REFERENCE_DIR)")
    args = ap.parse_args()
    if not args.reference_dir:
        ap.error("give --reference-dir or set BPT_REFERENCE_DIR")
    ref = load_reference(args.reference_dir)
    import torch
    torch.set_num_threads(os.cpu_count() or 1)

    arrays, meta = {}, []
    for spec in fp16_specs():
        c = build_fp16(spec)
        out = run_reference(ref, c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                            c["seq_lens"])
        spec["digest"] = oc.digest(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                   c["seq_lens"])
        arrays[spec["name"] + "/out"] = out.astype(np.float16)
        meta.append(spec)
        print("fp16", spec["name"], out.shape)
    for spec in quant_specs():
        c = build_quant(spec)
        kd, vd = kivi.dequantize_cache(c["cache"], spec["fmt"])
        # the reference casts its result to q.dtype; q is fp16 here
        out = run_reference(ref, c["q"], kd, vd, c["block_table"], c["seq_lens"])
        spec["digest"] = quant_digest(c)
        arrays[spec["name"] + "/out"] = out.astype(np.float16)
        meta.append(spec)
        print("quant", spec["name"], out.shape)
    for spec in code_specs():
        c = build_quant(spec, garbage=False)
        spec["digest"] = oc.digest(c["k"], c["v"], c["block_table"], c["seq_lens"])
        for k, a in c["cache"].items():
            arrays[spec["name"] + "/" + k] = a
        meta.append(spec)
        print("codes", spec["name"])
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(dict(generator="tests/golden/make_golden.py",
                       reference="src/bpt/reference.py:paged_decode_attention_ref",
                       cases=meta), f, indent=1)


if __name__ == "__main__":
    main()
