"""Fused sequence-shard exchange kernel (bpt_seqx_merge_fp16) on one GPU.

* world 1: the fused split merge + rank merge equals the plain split merge (merge_partials);
  repeated calls (fresh epochs) and a CUDA-graph replay give the same result.
* a failed peer without a fault: a world-2 exchange whose second "rank" is this rank's own
  buffer never receives rank 1's flags, so the kernel's bounded wait must run out, report
  BPT_DEV_WAIT_TIMEOUT in the status word and return; the context stays usable.
The multi-GPU exchange itself is covered by tests/test_dist_gpu.py.
"""
import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _partials(B=2, Hq=32, S=9, D=128, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    o = torch.randn(B, Hq, S, D, generator=g, device="cuda")
    lse = torch.randn(B, Hq, S, generator=g, device="cuda") * 4
    lse[0, :, 3] = float("-inf")          # an empty split
    o[0, :, 3] = float("nan")             # ... whose row is never read
    return o, lse


def _buffer(world, B, Hq, D):
    from bpt.dist import IPC_HANDLE_BYTES, _seqx_fns
    f = _seqx_fns()
    buf = ctypes.c_void_p()
    h = (ctypes.c_char * IPC_HANDLE_BYTES)()
    rc = f["alloc"](f["bytes"](world, B, Hq, D), ctypes.byref(buf), ctypes.cast(h, ctypes.c_void_p))
    assert rc == 0
    return buf.value


def _merge(o, lse, bufs, rank, status, out, budget_us=2_000_000):
    from bpt.dist import _seqx_fns
    B, Hq, S, D = o.shape
    arr = (ctypes.c_void_p * len(bufs))(*bufs)
    return _seqx_fns()["merge"](o.data_ptr(), lse.data_ptr(), B, Hq, D, S,
                                ctypes.cast(arr, ctypes.c_void_p), len(bufs), rank,
                                out.data_ptr(), out.stride(0), out.stride(1), status.data_ptr(),
                                budget_us, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("S,D", [(9, 128), (200, 128), (74, 256), (130, 64)])
def test_world1_equals_split_merge_and_replays(S, D):
    """S > 128 takes more than one batch of split rows per warp; D = 256 two channel groups."""
    from bpt.decode import merge_partials
    from bpt.dist import _seqx_fns
    o, lse = _partials(S=S, D=D)
    B, Hq, S, D = o.shape
    ref = merge_partials(o, lse)
    buf = _buffer(1, B, Hq, D)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty(B, Hq, D, dtype=torch.float16, device="cuda")
    for _ in range(3):
        out.zero_()
        assert _merge(o, lse, [buf], 0, status, out) == 0
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert (out.float() - ref.float()).abs().max().item() <= 2e-3
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            _merge(o, lse, [buf], 0, status, out)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert (out.float() - ref.float()).abs().max().item() <= 2e-3
    assert int(status.item()) == 0
    del g
    _seqx_fns()["free"](buf)


def test_missing_peer_times_out_and_reports():
    from bpt import paged_decode_attention
    from bpt.cache import random_paged_workload
    from bpt.dist import _seqx_fns
    o, lse = _partials(B=1)
    B, Hq, S, D = o.shape
    buf = _buffer(2, B, Hq, D)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty(B, Hq, D, dtype=torch.float16, device="cuda")
    t0 = time.perf_counter()
    assert _merge(o, lse, [buf, buf], 0, status, out, budget_us=20000) == 0
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert int(status.item()) & 4, "BPT_DEV_WAIT_TIMEOUT not reported"
    assert 0.015 < waited < 5.0, waited
    _seqx_fns()["free"](buf)
    w = random_paged_workload([300], 32, 8, 128, 16, "cuda", seed=3)   # the GPU still works
    r = paged_decode_attention(w["q"], w["k_cache"], w["v_cache"], w["block_table"],
                               w["seq_lens"])
    torch.cuda.synchronize()
    assert torch.isfinite(r.float()).all()
