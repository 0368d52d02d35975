"""FP16 decode kernel parity on the GPU (B200).

Mirrors the reference's tests/test_triton_fp16.py: the same shape list, block sizes, ragged
lengths and num_splits values (1, 2, 3, 7 -> some splits empty, None -> heuristic), bitwise
determinism and split invariance -- checked against the reference's own outputs (golden
fixtures made by tests/golden/make_golden.py) and the CPU oracle, at the BASELINE tolerance
(max abs 2e-3, max rel 1e-2 with the reference's clamp_min(1e-3)). Adds: empty sequences,
NaN garbage in unused slots, strided / head-major cache views, CUDA-graph capture, argument
errors, device-side checks, and a full-size ragged batch against a torch fp32 reference.
"""
import functools

import numpy as np
import pytest
import torch

from helpers import assert_close, build_fp16, golden_arrays, golden_meta, torch_reference

pytestmark = pytest.mark.gpu

FP16_CASES = [c for c in golden_meta() if c["kind"] == "fp16"]
SPLITS = [1, 2, 3, 7, None]


@functools.lru_cache(maxsize=None)
def _case(name):
    spec = next(c for c in FP16_CASES if c["name"] == name)
    return spec, build_fp16(spec)


@functools.lru_cache(maxsize=None)
def _oracle(name):
    from oracle import attention as oa
    _, c = _case(name)
    return oa.paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                         c["seq_lens"])


def _to_gpu(c):
    return (torch.from_numpy(c["q"]).cuda(), torch.from_numpy(c["k_cache"]).cuda(),
            torch.from_numpy(c["v_cache"]).cuda(), torch.from_numpy(c["block_table"]).cuda(),
            torch.from_numpy(c["seq_lens"]).cuda())


@pytest.mark.parametrize("num_splits", SPLITS)
@pytest.mark.parametrize("name", [c["name"] for c in FP16_CASES])
def test_matches_reference(name, num_splits):
    from bpt import paged_decode_attention
    spec, c = _case(name)
    out = paged_decode_attention(*_to_gpu(c), num_splits=num_splits)
    out = out.cpu().numpy()
    assert_close(out, golden_arrays()[name + "/out"], what=f"{name} vs reference")
    assert_close(out, _oracle(name), what=f"{name} vs oracle")


def test_reference_entry_point_name():
    from bpt.triton_fp16 import paged_decode_attention_triton
    spec, c = _case("c1")
    out = paged_decode_attention_triton(*_to_gpu(c))
    assert_close(out.cpu().numpy(), golden_arrays()["c1/out"])


def test_split_kv_is_deterministic():
    from bpt import paged_decode_attention
    _, c = _case("fp16_h32_8_d128_bs16_l4096-1000-17-2049")
    args = _to_gpu(c)
    a = paged_decode_attention(*args, num_splits=8)
    b = paged_decode_attention(*args, num_splits=8)
    assert torch.equal(a, b)


def test_splits_agree_with_single_pass():
    from bpt import paged_decode_attention
    _, c = _case("fp16_h32_8_d128_bs32_l4096-1000-17-2049")
    args = _to_gpu(c)
    base = paged_decode_attention(*args, num_splits=1)
    for n in (2, 5, 16, 64):
        out = paged_decode_attention(*args, num_splits=n)
        assert (out.float() - base.float()).abs().max().item() < 2e-3


def test_nan_garbage_is_never_read():
    """Unused slots and pages full of NaN must not leak into the result."""
    from bpt import paged_decode_attention
    name = "fp16_h32_8_d128_bs16_l100-33-1-64"
    spec, c = _case(name)
    kc, vc = c["k_cache"].copy(), c["v_cache"].copy()
    bs = spec["block_size"]
    used = np.zeros(kc.shape[:2], dtype=bool)
    for b, n in enumerate(spec["lens"]):
        for t in range(n):
            used[c["block_table"][b, t // bs], t % bs] = True
    kc[~used] = np.nan
    vc[~used] = np.nan
    q, _, _, bt, sl = _to_gpu(c)
    for ns in (1, 3, None):
        out = paged_decode_attention(q, torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda(),
                                     bt, sl, num_splits=ns).cpu().numpy()
        assert_close(out, golden_arrays()[name + "/out"], what=f"nan garbage splits={ns}")


def test_strided_and_head_major_caches():
    """k/v as views of one [nb, 2, bs, Hkv, D] allocation, and a head-major page layout."""
    from bpt import paged_decode_attention
    name = "fp16_h32_8_d128_bs16_l4096-1000-17-2049"
    _, c = _case(name)
    q, kc, vc, bt, sl = _to_gpu(c)
    kv = torch.stack([kc, vc], dim=1)                      # [nb, 2, bs, H, D]
    out = paged_decode_attention(q, kv[:, 0], kv[:, 1], bt, sl)
    assert_close(out.cpu().numpy(), golden_arrays()[name + "/out"], what="interleaved kv")
    kh = kc.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)  # storage [nb, H, bs, D]
    vh = vc.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)
    out = paged_decode_attention(q, kh, vh, bt, sl, num_splits=4)
    assert_close(out.cpu().numpy(), golden_arrays()[name + "/out"], what="head-major pages")


def test_cuda_graph_capture_and_replay():
    from bpt import paged_decode_attention
    _, c = _case("c1")
    args = _to_gpu(c)
    ref = paged_decode_attention(*args)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        paged_decode_attention(*args)  # warm-up on the side stream
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = paged_decode_attention(*args)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_argument_errors_match_reference_asserts():
    from bpt import BptArgumentError, paged_decode_attention
    _, c = _case("c1")
    q, kc, vc, bt, sl = _to_gpu(c)
    with pytest.raises(AssertionError):
        paged_decode_attention(q.float(), kc, vc, bt, sl)         # not fp16
    with pytest.raises(AssertionError):
        paged_decode_attention(q, kc, vc, bt.long(), sl)          # int64 table
    with pytest.raises(BptArgumentError):
        paged_decode_attention(q[:, :30], kc, vc, bt, sl)         # 30 % 8 != 0
    with pytest.raises(ValueError):
        paged_decode_attention(q.cpu(), kc, vc, bt, sl)           # no CPU fallback


def test_device_check_flags_bad_block_id(monkeypatch):
    """A block id outside [0, num_blocks) is caught by the kernel's own check (it is clamped
    before use) and reported in checked mode."""
    import bpt.decode as dec
    from bpt import BptError
    _, c = _case("c1")
    q, kc, vc, bt, sl = _to_gpu(c)
    bad = bt.clone()
    bad[0, 3] = kc.shape[0] + 5
    monkeypatch.setattr(dec, "CHECKS", True)
    with pytest.raises(BptError, match="block_table"):
        dec.paged_decode_attention(q, kc, vc, bad, sl)
    dec.paged_decode_attention(q, kc, vc, bt, sl)  # clean call passes in checked mode


def test_bounded_wait_gives_up_and_reports_timeout():
    """Failure detection without a fault: a CTA waits (through the decode kernels' bounded
    wait) on a barrier phase nothing completes; after its 50 ms budget it must return and
    report BPT_DEV_WAIT_TIMEOUT in the status word, and the context must stay usable."""
    import time
    from bpt import _lib, paged_decode_attention
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    rc = _lib.lib().bpt_selftest_wait_timeout(status.data_ptr(), 50000, stream)
    _lib.check(rc, "bpt_selftest_wait_timeout")
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert int(status.item()) & 4, "BPT_DEV_WAIT_TIMEOUT not reported"
    assert 0.04 < waited < 5.0, waited
    _, c = _case("c1")
    out = paged_decode_attention(*_to_gpu(c))           # the context still works
    assert_close(out.cpu().numpy(), golden_arrays()["c1/out"], what="after the timeout")


@pytest.mark.parametrize("D", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("Hq,Hkv", [(8, 8), (16, 8), (32, 8), (16, 2)])   # groups 1, 2, 4, 8
@pytest.mark.parametrize("bs", [16, 256])
def test_head_dims_groups_and_page_sizes(D, Hq, Hkv, bs):
    """Every head_dim the kernels are built for (CUDA-core kernel for 16/32, tensor-core for
    64/128/256) x groups 1-8 x the smallest and largest page size, ragged lengths with a
    one-token and a page-crossing sequence, against the numpy oracle."""
    from bpt import paged_decode_attention
    from oracle import attention as oa
    from oracle import cache as oc
    lens = [1, bs + 3, 3 * bs - 1]
    c = oc.fp16_case(100 + D + Hq + bs, lens, Hq, Hkv, D, bs, "reference", 8)
    ref = oa.paged_decode_attention_ref(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                        c["seq_lens"])
    for ns in (1, 3, None):
        out = paged_decode_attention(*_to_gpu(c), num_splits=ns)
        assert_close(out.cpu().numpy(), ref, what=f"D={D} Hq={Hq} Hkv={Hkv} bs={bs} ns={ns}")


@pytest.mark.parametrize("B,ctx", [(8, 16384), (1, 65536)])
def test_full_size_batch_against_torch_fp32(B, ctx):
    """BASELINE FP16 shapes (ragged U[0.75 ctx, ctx], bs=16) against a torch fp32 reference."""
    from bpt import paged_decode_attention
    from bpt.cache import ragged_lengths, random_paged_workload
    lens = ragged_lengths(B, ctx, seed=11) if B > 1 else [ctx]
    w = random_paged_workload(lens, 32, 8, 128, 16, "cuda", seed=11, spare_blocks=64)
    ref = torch_reference(w["q"], w["k_cache"], w["v_cache"], w["block_table"], w["seq_lens"])
    for ns in (None, 1):
        out = paged_decode_attention(w["q"], w["k_cache"], w["v_cache"], w["block_table"],
                                     w["seq_lens"], num_splits=ns)
        assert_close(out.float().cpu().numpy(), ref.cpu().numpy(), what=f"B={B} ctx={ctx}")


def test_balanced_splits_of_a_very_ragged_batch():
    """A batch launched as one wave cuts its LONGEST sequence into the splits and gives each
    shorter sequence only the splits that cover it (empty trailing splits, lse = -inf), so no
    CTA runs longer than another. Lengths from 0 to 16384 tokens, including one shorter than a
    chunk, at the planner's count and at explicit counts (all one wave for B=8)."""
    from bpt import paged_decode_attention
    from bpt.cache import random_paged_workload
    from bpt.decode import _sm_count, effective_splits
    lens = [16384, 1, 0, 16, 9000, 33, 16383, 4096]
    w = random_paged_workload(lens, 32, 8, 128, 16, "cuda", seed=21, spare_blocks=64)
    ref = torch_reference(w["q"], w["k_cache"], w["v_cache"], w["block_table"], w["seq_lens"])
    mb = w["block_table"].shape[1]
    assert effective_splits(8, 8, 16, mb, None, _sm_count(0)) * 8 * 8 <= 4 * _sm_count(0)
    for ns in (None, 2, 5, 9):
        out = paged_decode_attention(w["q"], w["k_cache"], w["v_cache"], w["block_table"],
                                     w["seq_lens"], num_splits=ns)
        assert torch.isfinite(out.float()).all()
        assert_close(out.float().cpu().numpy(), ref.cpu().numpy(), what=f"splits={ns}")
        assert out[2].abs().max().item() == 0.0   # the empty sequence gives zeros


@pytest.mark.parametrize("splits", [1, 4, 9])
def test_partial_states_and_merges(splits):
    """bpt_decode_fp16_partial + bpt_merge_states give the oracle's per-sequence state
    (o, lse); lse is reported in log2 units."""
    from bpt.decode import merge_partials, merge_states, paged_decode_attention_partial
    from oracle import attention as oa
    name = "fp16_h32_8_d128_bs16_l4096-1000-17-2049"
    spec, c = _case(name)
    q, kc, vc, bt, sl = _to_gpu(c)
    o_part, lse = paged_decode_attention_partial(q, kc, vc, bt, sl, num_splits=splits)
    assert o_part.shape[2] == splits
    out = merge_partials(o_part, lse)
    assert_close(out.cpu().numpy(), golden_arrays()[name + "/out"], what="merge_partials")
    o, l2 = merge_states(o_part, lse)
    lens = c["seq_lens"]
    o_ref, lse_ref = oa.paged_decode_attention_partial(
        c["q"], c["k_cache"], c["v_cache"], c["block_table"], lens, np.zeros_like(lens), lens)
    assert np.abs(o.cpu().numpy() - o_ref).max() < 1e-4
    assert np.abs(l2.cpu().numpy() - lse_ref * np.log2(np.e)).max() < 1e-4


def test_long_biased_values_single_split():
    """128k tokens of V ~ N(5, 1) in ONE split: every warp accumulates 64k tokens of positive
    contributions in a single tensor-core accumulator; the result must stay within tolerance."""
    from bpt import paged_decode_attention
    from bpt.cache import random_paged_workload
    w = random_paged_workload([131072], 32, 8, 128, 16, "cuda", seed=21)
    w["v_cache"].add_(5.0)
    ref = torch_reference(w["q"], w["k_cache"], w["v_cache"], w["block_table"], w["seq_lens"])
    for ns in (1, None):
        out = paged_decode_attention(w["q"], w["k_cache"], w["v_cache"], w["block_table"],
                                     w["seq_lens"], num_splits=ns)
        assert_close(out.float().cpu().numpy(), ref.cpu().numpy(), what=f"biased V ns={ns}")
