"""bpt_decode_fp16_noalloc: decode for callers that cannot allocate device memory.

Some callers cannot call cudaMalloc when they run decode (an engine that owns all device
memory after start-up, a plugin handed only its input and output buffers). They use
bpt_decode_fp16_noalloc, which keeps the split partial states in a fixed scratch array inside
the library instead of a caller workspace. These tests call it through the C ABI and check:

* two calls in a row (so leftover scratch contents from the first call cannot leak into the
  second) against bpt_decode_fp16 (reached through bpt.paged_decode_attention), against the
  reference's own outputs (golden fixtures) and against the numpy oracle, at the tolerance
  every parity test here uses;
* a second call of the SAME shape over a scratch array already full of the first call's data,
  with shorter and zero sequence lengths, so some splits are empty and the merge must not read
  stale partial rows;
* what a caller of this no-status path gets for an out-of-range block id: rc 0 and a finite
  output equal to bpt_decode_fp16's on the same input (both kernels read page 0 instead);
* that an oversized call is refused without a launch.

This file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import assert_close, build_fp16, golden_arrays, golden_meta

pytestmark = pytest.mark.gpu

c_i32, c_i64, c_f32, c_vp = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p
ARGTYPES = [c_vp, c_i64, c_i64,
            c_vp, c_i64, c_i64, c_i64,
            c_vp, c_i64, c_i64, c_i64,
            c_i64, c_vp, c_i64, c_vp,
            c_vp, c_i64, c_i64,
            c_i32, c_i32, c_i32, c_i32, c_i32, c_i32,
            c_f32, c_i32, c_i32, c_vp]
SCRATCH_BYTES = 8 * 1024 * 1024  # BPT_NOALLOC_SCRATCH_BYTES in include/bpt.h


def _noalloc_fn():
    from bpt import _lib
    return _lib.register("bpt_decode_fp16_noalloc", c_i32, ARGTYPES)


def _call_noalloc(q, kc, vc, bt, sl, num_splits):
    from bpt.decode import _sm_count
    out = torch.full_like(q, float("nan"))
    rc = _noalloc_fn()(
        q.data_ptr(), q.stride(0), q.stride(1),
        kc.data_ptr(), kc.stride(0), kc.stride(1), kc.stride(2),
        vc.data_ptr(), vc.stride(0), vc.stride(1), vc.stride(2), kc.shape[0],
        bt.data_ptr(), bt.stride(0), sl.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1),
        q.shape[0], q.shape[1], kc.shape[2], q.shape[2], kc.shape[1], bt.shape[1],
        0.0, num_splits, _sm_count(q.device.index or 0),
        torch.cuda.current_stream().cuda_stream)
    return rc, out


def _case(name):
    spec = next(c for c in golden_meta() if c["name"] == name)
    return build_fp16(spec)


def _to_gpu(c):
    return [torch.from_numpy(c[k]).cuda() for k in
            ("q", "k_cache", "v_cache", "block_table", "seq_lens")]


def _oracle(c, seq_lens=None, block_table=None):
    from oracle import attention as oa
    return oa.paged_decode_attention_ref(
        c["q"], c["k_cache"], c["v_cache"],
        c["block_table"] if block_table is None else block_table,
        c["seq_lens"] if seq_lens is None else seq_lens)


def test_noalloc_matches_workspace_entry_point_on_two_calls_in_a_row():
    from bpt import paged_decode_attention
    from bpt.decode import _sm_count, effective_splits
    cases = [("c1", 0), ("fp16_h32_8_d128_bs16_l4096-1000-17-2049", 7)]
    for name, ns in cases:
        c = _case(name)
        q, kc, vc, bt, sl = _to_gpu(c)
        S = effective_splits(q.shape[0], kc.shape[2], kc.shape[1], bt.shape[1], ns,
                             _sm_count(0))
        assert S > 1, "the case must exercise the scratch (several splits)"
        rc, out = _call_noalloc(q, kc, vc, bt, sl, ns)
        torch.cuda.synchronize()
        assert rc == 0, rc
        got = out.float().cpu().numpy()
        ref = paged_decode_attention(q, kc, vc, bt, sl, num_splits=ns or None)
        assert_close(got, ref.float().cpu().numpy(), what=f"noalloc vs bpt_decode_fp16 ({name})")
        assert_close(got, golden_arrays()[name + "/out"], what=f"noalloc vs reference ({name})")
        assert_close(got, _oracle(c), what=f"noalloc vs oracle ({name})")


def test_noalloc_same_shape_second_call_with_shorter_and_empty_sequences():
    """The first call fills the scratch rows of every split; the second, same shape and split
    count, has shorter and zero-length sequences, so some of its splits are empty. Its result
    must equal the oracle on the new lengths: no stale partial row may be merged."""
    from bpt import paged_decode_attention
    name = "fp16_h32_8_d128_bs16_l4096-1000-17-2049"
    c = _case(name)
    q, kc, vc, bt, sl = _to_gpu(c)
    ns = 9
    rc, out = _call_noalloc(q, kc, vc, bt, sl, ns)
    torch.cuda.synchronize()
    assert rc == 0, rc
    assert_close(out.float().cpu().numpy(), golden_arrays()[name + "/out"], what="first call")
    short = np.asarray([700, 0, 17, 1], dtype=np.int32)    # vs [4096, 1000, 17, 2049]
    sl2 = torch.from_numpy(short).cuda()
    rc, out2 = _call_noalloc(q, kc, vc, bt, sl2, ns)
    torch.cuda.synchronize()
    assert rc == 0, rc
    got = out2.float().cpu().numpy()
    assert_close(got, _oracle(c, seq_lens=short), what="second call vs oracle")
    assert np.all(got[1] == 0.0), "an empty sequence gives zeros"
    ref = paged_decode_attention(q, kc, vc, bt, sl2, num_splits=ns)
    assert_close(got, ref.float().cpu().numpy(), what="second call vs bpt_decode_fp16")


def test_noalloc_out_of_range_block_id_reads_page_zero():
    """This path has no status word: an out-of-range block id is not reported. The kernels
    clamp it to page 0 before reading, so the caller gets rc 0 and the finite result of that
    substitution, the same as bpt_decode_fp16 gives (which also flags it in its workspace)."""
    from bpt import paged_decode_attention
    c = _case("c1")
    q, kc, vc, bt, sl = _to_gpu(c)
    bad = c["block_table"].copy()
    bad[0, 3] = kc.shape[0] + 5
    bad_gpu = torch.from_numpy(bad).cuda()
    rc, out = _call_noalloc(q, kc, vc, bad_gpu, sl, 0)
    torch.cuda.synchronize()
    assert rc == 0, rc
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    ref = paged_decode_attention(q, kc, vc, bad_gpu, sl)
    assert_close(got, ref.float().cpu().numpy(), what="bad block id vs bpt_decode_fp16")
    substituted = c["block_table"].copy()
    substituted[0, 3] = 0
    assert_close(got, _oracle(c, block_table=substituted), what="bad block id vs oracle(page 0)")


def test_noalloc_refuses_more_scratch_than_it_has():
    from bpt import _lib
    B, Hq, Hkv, D, bs, max_blocks, splits = 64, 32, 8, 128, 16, 256, 64
    need = 256 + B * Hq * splits * 4 + B * Hq * splits * D * 4
    assert need > SCRATCH_BYTES
    q = torch.zeros(B, Hq, D, dtype=torch.float16, device="cuda")
    kc = torch.zeros(4, bs, Hkv, D, dtype=torch.float16, device="cuda")
    bt = torch.zeros(B, max_blocks, dtype=torch.int32, device="cuda")
    sl = torch.zeros(B, dtype=torch.int32, device="cuda")
    rc, out = _call_noalloc(q, kc, kc, bt, sl, splits)
    assert rc == _lib.ERR_WORKSPACE_TOO_SMALL
    assert torch.isnan(out).all(), "a refused call must not launch"
