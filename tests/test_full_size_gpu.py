"""Full-size parity at every BASELINE configuration (GPU).

The golden fixtures pin the kernels at sizes the CPU oracle finishes in seconds; these tests
run the BASELINE configurations themselves and check sampled sequences (every q head of the
first, the last and two seeded random sequences) against an fp32 torch restatement of the
reference oracle (src/bpt/reference.py:20-49) on the GPU, at the BASELINE tolerance (max abs
2e-3, max rel 1e-2 with the reference's clamp_min(1e-3)):

* FP16, B in {8, 16, 32, 64} x ctx in {16k, 64k}, seq_len ~ U[0.75 ctx, ctx],
  block_size 16, random-permutation block tables;
* FP16, B = 1 at 4k, 16k, 64k and 128k tokens, q, K, V ~ N(0, 1);
* INT8 and FP8-E4M3 KIVI, block_size 64, K ~ N(0, 1) with 4 seeded x10 outlier
  channels per kv head, V ~ N(0, 1), B in {1, 8, 32} x ctx in {8k, 32k, 128k}, quantized on the
  GPU by the append kernel and checked against fp32 attention on the dequantized cache;
* INT4 KIVI with the same distribution at B=64/32k and B=1/128k (plus B=8/8k and
  B=32/32k).

Each case runs the planner's split count and one or two forced ones (a single pass at B=1, so
one CTA per kv head streams the whole sequence).
"""
import pytest
import torch

from helpers import assert_close, sample_seqs, torch_reference, torch_reference_kivi

pytestmark = pytest.mark.gpu

HQ, HKV, D = 32, 8, 128


def _lens(B, ctx, seed):
    from bpt.cache import ragged_lengths
    return ragged_lengths(B, ctx, seed=seed) if B > 1 else [ctx]


def _check(out, ref, seqs, what):
    assert_close(out[seqs].float().cpu().numpy(), ref.cpu().numpy(), what=what)


@pytest.mark.parametrize("ctx", [16384, 65536])
@pytest.mark.parametrize("B", [8, 16, 32, 64])
def test_fp16_batch(B, ctx):
    from bpt import paged_decode_attention
    from bpt.cache import random_paged_workload
    lens = _lens(B, ctx, seed=B + ctx)
    w = random_paged_workload(lens, HQ, HKV, D, 16, "cuda", seed=B * 7 + 1, spare_blocks=64)
    seqs = sample_seqs(B, 4, seed=B)
    ref = torch_reference(w["q"], w["k_cache"], w["v_cache"], w["block_table"], w["seq_lens"],
                          seqs=seqs)[seqs]
    for ns in (None, 5):
        out = paged_decode_attention(w["q"], w["k_cache"], w["v_cache"], w["block_table"],
                                     w["seq_lens"], num_splits=ns)
        _check(out, ref, seqs, f"fp16 B={B} ctx={ctx} splits={ns}")


@pytest.mark.parametrize("ctx", [4096, 16384, 65536, 131072])
def test_fp16_batch1(ctx):
    from bpt import paged_decode_attention
    from bpt.cache import random_paged_workload
    w = random_paged_workload([ctx], HQ, HKV, D, 16, "cuda", seed=ctx % 1000 + 3,
                              spare_blocks=64)
    ref = torch_reference(w["q"], w["k_cache"], w["v_cache"], w["block_table"], w["seq_lens"])
    for ns in (None, 1, 7):
        out = paged_decode_attention(w["q"], w["k_cache"], w["v_cache"], w["block_table"],
                                     w["seq_lens"], num_splits=ns)
        _check(out, ref, [0], f"fp16 B=1 ctx={ctx} splits={ns}")


KIVI_CASES = ([(f, B, ctx) for f in ("int8", "fp8") for B in (1, 8, 32)
               for ctx in (8192, 32768, 131072)]
              + [("int4", 1, 131072), ("int4", 64, 32768), ("int4", 8, 8192),
                 ("int4", 32, 32768)])


@pytest.mark.parametrize("fmt,B,ctx", KIVI_CASES)
def test_kivi_outlier_keys(fmt, B, ctx):
    """The BASELINE KIVI distribution: 4 seeded x10 outlier key channels per kv head (the case
    the fixed-point headroom of the integer kernels is sized for)."""
    from bpt.quant import paged_decode_attention_kivi, random_kivi_workload
    lens = _lens(B, ctx, seed=B + ctx + 1)
    w = random_kivi_workload(lens, HQ, HKV, D, 64, fmt, "cuda", seed=B * 13 + ctx % 997,
                             outlier_channels=4, outlier_scale=10.0, spare_blocks=16)
    seqs = sample_seqs(B, 4, seed=B + 1)
    ref = torch_reference_kivi(w["q"], w["cache"], w["block_table"], w["seq_lens"], seqs)
    for ns in ((None, 1, 7) if B == 1 else (None, 3)):
        out = paged_decode_attention_kivi(w["q"], w["cache"], w["block_table"], w["seq_lens"],
                                          num_splits=ns)
        _check(out, ref, seqs, f"{fmt} B={B} ctx={ctx} splits={ns}")
    del w
    torch.cuda.empty_cache()
