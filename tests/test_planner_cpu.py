"""Split planner invariants through the C ABI (bpt_plan_splits), over random shapes (CPU only:
the planner is host code).

* 1 <= splits <= max(1, chunks / 2) (a split is at least 2 chunks of 32 tokens);
* a one-wave plan (at least 4 splits fit in one wave of 4 CTAs per SM) is taken exactly when
  its splits stay at most 8192 tokens of the table long;
* otherwise the plan has at most just under 7 full waves, and splits of at least 1024 tokens
  unless that would leave less than one wave.
"""
import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings, strategies as st  # noqa: E402

CHUNK = 32
RESIDENT = 4


def _plan(batch, kv_heads, block_size, max_blocks, sms):
    from bpt.decode import choose_num_splits
    return choose_num_splits(batch, kv_heads, block_size, max_blocks, sms)


@settings(max_examples=400, deadline=None)
@given(batch=st.integers(1, 1024), kv_heads=st.sampled_from([1, 2, 4, 8, 16]),
       block_size=st.sampled_from([16, 32, 64, 128, 256]), tokens=st.integers(1, 1 << 21),
       sms=st.sampled_from([1, 16, 132, 148, 160]))
def test_planner_invariants(batch, kv_heads, block_size, tokens, sms):
    max_blocks = -(-tokens // block_size)
    s = _plan(batch, kv_heads, block_size, max_blocks, sms)
    units = -(-(max_blocks * block_size) // CHUNK)
    assert 1 <= s <= max(1, units // 2)
    work = batch * kv_heads
    resident = sms * RESIDENT
    one_wave = resident // work
    span = units * CHUNK
    if one_wave >= 4 and span <= 8192 * one_wave:
        assert s == min(one_wave, max(1, units // 2))
    else:
        assert s <= max(1, 7 * resident // work, one_wave)
        if s > max(one_wave, 1) and s < max(1, units // 2):
            assert span // s >= 1024


def test_planner_examples_on_b200():
    # one wave at B=1 (74 x 8 = 592 CTAs), several waves for long single-wave splits
    assert _plan(1, 8, 16, 8192, 148) == 74          # 128k tokens: 1771 tokens per split
    assert _plan(8, 8, 16, 4096, 148) == 9           # 64k, 7282 tokens per split: one wave
    assert _plan(8, 8, 16, 8192, 148) == 64          # 128k: 14.6k per split -> 7 waves
    assert _plan(64, 8, 16, 1024, 148) == 8          # 7 waves of 512 work items
