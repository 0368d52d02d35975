"""bpt's FlashInfer-compatible decode wrapper against FlashInfer's own
BatchDecodeWithPagedKVCacheWrapper (the library installed in this image), same inputs, same
GPU: NHD and HND layouts, stacked and (k, v)-tuple caches, ragged batches with partial last
pages and an empty sequence, groups 1-8, page sizes 16 / 64; outputs within the BASELINE
absolute tolerance of each other and of a torch fp32 reference; the returned log-sum-exp
(base 2) against FlashInfer's."""
import math

import pytest
import torch

from helpers import ATOL

pytestmark = pytest.mark.gpu
flashinfer = pytest.importorskip("flashinfer")


def _case(lens, Hq, Hkv, D, ps, layout, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    pages = [(n + ps - 1) // ps for n in lens]
    P = sum(pages) + 7
    shape = (P, 2, ps, Hkv, D) if layout == "NHD" else (P, 2, Hkv, ps, D)
    kv = torch.randn(shape, generator=g, device="cuda", dtype=torch.float16)
    perm = torch.randperm(P, generator=torch.Generator().manual_seed(seed))[:sum(pages)]
    indices = perm.to(torch.int32).cuda()
    indptr = torch.tensor([0] + list(torch.tensor(pages).cumsum(0)), dtype=torch.int32,
                          device="cuda")
    last = torch.tensor([(n - 1) % ps + 1 if n else 0 for n in lens], dtype=torch.int32,
                        device="cuda")
    q = torch.randn(len(lens), Hq, D, generator=g, device="cuda", dtype=torch.float16)
    return q, kv, indptr, indices, last


@pytest.mark.parametrize("layout", ["NHD", "HND"])
@pytest.mark.parametrize("Hq,Hkv,D,ps", [(32, 8, 128, 16), (32, 8, 128, 64), (16, 2, 128, 16),
                                         (8, 8, 64, 16)])
def test_matches_flashinfer(layout, Hq, Hkv, D, ps):
    from bpt.flashinfer_compat import BatchDecodeWithPagedKVCacheWrapper
    lens = [1, 37, 4096, 2731, ps * 3]
    q, kv, indptr, indices, last = _case(lens, Hq, Hkv, D, ps, layout, seed=Hq + D + ps)
    ws = torch.empty(128 << 20, dtype=torch.uint8, device="cuda")
    fi = flashinfer.BatchDecodeWithPagedKVCacheWrapper(ws, layout)
    fi.plan(indptr, indices, last, Hq, Hkv, D, ps, q_data_type=torch.float16,
            kv_data_type=torch.float16)
    want, want_lse = fi.run(q, kv, return_lse=True)
    ours = BatchDecodeWithPagedKVCacheWrapper(torch.empty(64 << 20, dtype=torch.uint8,
                                                          device="cuda"), layout)
    ours.plan(indptr, indices, last, Hq, Hkv, D, ps)
    got = ours.run(q, kv)
    got_t = ours.run(q, (kv[:, 0], kv[:, 1]))
    got2, lse2 = ours.run(q, kv, return_lse=True)
    torch.cuda.synchronize()
    d = (got.float() - want.float()).abs().max().item()
    assert d < ATOL, f"vs FlashInfer: max abs {d:.3e}"
    assert torch.equal(got, got_t) and (got2.float() - got.float()).abs().max().item() < 1e-3
    assert (lse2 - want_lse).abs().max().item() < 1e-3, "log-sum-exp (base 2) differs"
    # and both against fp32 attention computed directly from the pages
    from helpers import torch_reference
    k = kv[:, 0] if layout == "NHD" else kv[:, 0].transpose(1, 2)
    v = kv[:, 1] if layout == "NHD" else kv[:, 1].transpose(1, 2)
    ref = torch_reference(q, k, v, ours._bt, ours._sl)
    assert (got.float() - ref).abs().max().item() < ATOL


def test_empty_sequence_gives_zeros():
    from bpt.flashinfer_compat import BatchDecodeWithPagedKVCacheWrapper
    q, kv, indptr, indices, last = _case([100, 0, 5], 32, 8, 128, 16, "NHD")
    w = BatchDecodeWithPagedKVCacheWrapper(None, "NHD")
    w.plan(indptr, indices, last, 32, 8, 128, 16)
    out = w.run(q, kv)
    torch.cuda.synchronize()
    assert out[1].abs().max().item() == 0.0 and math.isfinite(out.float().abs().max().item())
