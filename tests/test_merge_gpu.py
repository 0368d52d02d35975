"""Split-merge kernel (bpt_merge_partials / bpt_merge_states) on the GPU against a float64
torch statement of the reference's merge (src/bpt/triton_fp16.py:152-162, in log2 units).

The kernel reads up to 128 split rows per CTA in one batch of loads and merges further rows
online; these cases cover one and several batches per warp (S up to 300), 1 to 8 warps, every
head_dim group layout (one or two 32-lane channel groups), the scalar path (head_dim not a
multiple of 4, or partials that do not start on a 16-byte boundary), empty splits whose rows
hold NaN, and sequences whose splits are all empty.
"""
import pytest
import torch

from helpers import assert_close

pytestmark = pytest.mark.gpu


def _partials(B, Hq, S, D, seed, all_empty_row=True):
    g = torch.Generator(device="cuda").manual_seed(seed)
    o = torch.randn(B, Hq, S, D, generator=g, device="cuda")
    lse = torch.randn(B, Hq, S, generator=g, device="cuda") * 6
    empty = torch.rand(B, Hq, S, generator=g, device="cuda") < 0.2
    lse[empty] = float("-inf")
    o[empty] = float("nan")               # rows of weight 0 are never used
    if all_empty_row:
        lse[0, 0] = float("-inf")         # a (sequence, head) with no tokens at all
        o[0, 0] = float("nan")
    return o, lse


def _reference(o, lse):
    o64, l64 = o.double(), lse.double()
    m = l64.max(-1, keepdim=True).values
    m_safe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    w = torch.exp2(l64 - m_safe)                        # 0 for -inf rows
    W = w.sum(-1)
    num = (torch.where(w[..., None] > 0, o64, torch.zeros_like(o64)) * w[..., None]).sum(-2)
    out = torch.where(W[..., None] > 0, num / W.clamp_min(1e-300)[..., None],
                      torch.zeros_like(num))
    lse_out = torch.where(W > 0, m_safe[..., 0] + torch.log2(W.clamp_min(1e-300)),
                          torch.full_like(W, float("-inf")))
    return out, lse_out


@pytest.mark.parametrize("S", [1, 2, 17, 74, 128, 129, 300])
@pytest.mark.parametrize("D", [16, 64, 128, 256])
def test_merge_matches_float64(S, D):
    from bpt.decode import merge_partials, merge_states
    B, Hq = 2, 8
    o, lse = _partials(B, Hq, S, D, seed=S * 1000 + D)
    ref_o, ref_l = _reference(o, lse)
    out = merge_partials(o, lse)
    assert_close(out.float().cpu().numpy(), ref_o.float().cpu().numpy(), what=f"S={S} D={D}")
    so, sl = merge_states(o, lse)
    assert torch.isfinite(so).all()
    assert (so.double() - ref_o).abs().max().item() < 1e-5
    fin = torch.isfinite(ref_l)
    assert torch.equal(torch.isfinite(sl), fin)
    assert (sl.double()[fin] - ref_l[fin]).abs().max().item() < 1e-5
    assert (out[0, 0] == 0).all() and so[0, 0].abs().max().item() == 0


@pytest.mark.parametrize("D", [18, 100])
def test_merge_scalar_path_head_dim(D):
    """head_dim not a multiple of 4 (D=18) or not a whole number of 32-lane groups (D=100)."""
    from bpt.decode import merge_partials
    o, lse = _partials(3, 4, 40, D, seed=D)
    out = merge_partials(o, lse)
    assert_close(out.float().cpu().numpy(), _reference(o, lse)[0].float().cpu().numpy(),
                 what=f"D={D}")


def test_merge_scalar_path_unaligned_partials():
    """Partials that start 4 bytes past a 16-byte boundary take the scalar-load path."""
    from bpt.decode import merge_partials
    B, Hq, S, D = 2, 8, 74, 128
    o, lse = _partials(B, Hq, S, D, seed=5)
    flat = torch.empty(o.numel() + 4, device="cuda")
    shifted = flat[1:1 + o.numel()].view(B, Hq, S, D)
    assert shifted.data_ptr() % 16 == 4 and shifted.is_contiguous()
    shifted.copy_(o)
    out = merge_partials(shifted, lse)
    assert_close(out.float().cpu().numpy(), _reference(o, lse)[0].float().cpu().numpy(),
                 what="unaligned")
    assert torch.equal(out, merge_partials(o, lse))   # same arithmetic order on both paths


def test_merge_is_deterministic():
    from bpt.decode import merge_partials
    o, lse = _partials(4, 32, 300, 128, seed=9)
    a = merge_partials(o, lse)
    for _ in range(3):
        assert torch.equal(a, merge_partials(o, lse))
