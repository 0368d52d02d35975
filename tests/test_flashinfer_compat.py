"""Host logic of the FlashInfer-compatible decode wrapper (CPU): CSR page lists -> block table
and sequence lengths, and the rejected FlashInfer features."""
import pytest
import torch


def _csr(pages_per_seq, last, seed=0):
    g = torch.Generator().manual_seed(seed)
    total = sum(pages_per_seq)
    indices = torch.randperm(total + 5, generator=g)[:total].to(torch.int32)
    indptr = torch.tensor([0] + list(torch.tensor(pages_per_seq).cumsum(0)), dtype=torch.int32)
    return indptr, indices, torch.tensor(last, dtype=torch.int32)


def test_csr_to_block_table_matches_a_plain_loop():
    from bpt.flashinfer_compat import csr_to_block_table
    pages = [3, 0, 1, 5]
    last = [7, 0, 16, 1]
    indptr, indices, lpl = _csr(pages, last)
    bt, sl = csr_to_block_table(indptr, indices, lpl, 16, "cpu")
    assert bt.dtype == sl.dtype == torch.int32 and bt.shape == (4, 5)
    for b, n in enumerate(pages):
        lo = int(indptr[b])
        assert bt[b, :n].tolist() == indices[lo:lo + n].tolist()
        assert int(sl[b]) == ((n - 1) * 16 + last[b] if n else 0)


def test_csr_edge_cases():
    from bpt.flashinfer_compat import csr_to_block_table
    bt, sl = csr_to_block_table(torch.tensor([0, 0, 0]), torch.zeros(0, dtype=torch.int32),
                                torch.zeros(2, dtype=torch.int32), 32, "cpu")
    assert bt.shape == (2, 1) and sl.tolist() == [0, 0]
    bt, sl = csr_to_block_table(torch.tensor([0]), torch.zeros(0, dtype=torch.int32),
                                torch.zeros(0, dtype=torch.int32), 16, "cpu")
    assert bt.shape == (0, 1) and sl.numel() == 0


def test_unsupported_features_are_rejected():
    from bpt import BptArgumentError
    from bpt.flashinfer_compat import BatchDecodeWithPagedKVCacheWrapper
    with pytest.raises(BptArgumentError):
        BatchDecodeWithPagedKVCacheWrapper(None, "NCHW")
    w = BatchDecodeWithPagedKVCacheWrapper(None, "NHD")
    indptr, indices, lpl = _csr([1], [3])
    for kw in (dict(pos_encoding_mode="ROPE_LLAMA"), dict(window_left=128),
               dict(logits_soft_cap=30.0), dict(kv_data_type=torch.float8_e4m3fn)):
        with pytest.raises(BptArgumentError):
            w.plan(indptr, indices, lpl, 32, 8, 128, 16, **kw)
