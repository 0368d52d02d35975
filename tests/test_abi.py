"""The C-ABI library loads on a CPU-only machine and exports every declared entry point;
host-only entry points (planner, workspace sizing, status strings) behave."""
import ctypes
import os
import re

import pytest

from bpt import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for fn in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", fn)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"\b(bpt_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "bpt_decode_fp16" in names and "bpt_plan_splits" in names


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports_symbol(name):
    lib = ctypes.CDLL(_lib.LIB_PATH)
    assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_status_strings():
    assert _lib.status_string(0) == "ok"
    assert "workspace" in _lib.status_string(-3)
    assert _lib.status_string(12345) == "unknown status"


def test_planner_fills_b200():
    from bpt.decode import choose_num_splits, effective_splits
    # B=1, 64k tokens, bs=16: one full wave of 4 CTAs/SM x 148 SMs (8 kv heads x 74 splits)
    assert choose_num_splits(1, 8, 16, 4096, 148) == 74
    # B=8: still one wave (64 x 9 = 576 <= 592), splits of at most 8192 tokens
    assert choose_num_splits(8, 8, 16, 1024, 148) == 9
    # B=64: fewer than 4 splits fit one wave -> just under 7 full waves (8 x 512 = 4096 CTAs)
    assert choose_num_splits(64, 8, 16, 4096, 148) == 8
    # B=16 at 64k: 4 splits would fit one wave but be 16k tokens long -> 7 waves (32 splits)
    assert choose_num_splits(16, 8, 16, 4096, 148) == 32
    # B=32 at 16k: 7 waves, splits of at least 1024 tokens
    assert choose_num_splits(32, 8, 16, 1024, 148) == 16
    # B=1 at 1M tokens: 74 splits would be 14k tokens long -> 7 waves of shorter ones
    assert choose_num_splits(1, 8, 16, 65536, 148) == 518
    # short context caps the split count (>= 2 chunks of 32 tokens per split)
    assert choose_num_splits(1, 8, 16, 16, 148) == 4
    assert choose_num_splits(1, 8, 16, 2, 148) == 1
    # explicit requests are clamped to the chunk count
    assert effective_splits(2, 8, 16, 4, 7, 148) == 2
    assert effective_splits(2, 8, 16, 512, 7, 148) == 7
    assert effective_splits(2, 8, 16, 512, 1, 148) == 1


def test_kivi_planner_uses_the_serving_kernels_shape():
    import ctypes
    from bpt import _lib
    f = _lib.register("bpt_effective_splits_kivi", ctypes.c_int, [ctypes.c_int] * 8)
    INT8, FP8, INT4 = 1, 2, 4 - 1
    # B=1, 128k tokens, bs=64, group 4: tcgen05 kernel, 128-token stages, 2 CTAs per SM
    # (148 x 2 / 8 kv heads = 37 splits)
    assert f(INT4, 1, 8, 32, 64, 2048, 0, 148) == 37
    assert f(INT8, 1, 8, 32, 64, 2048, 0, 148) == 37
    # 16-token pages: the mma.sync integer kernel (INT4: 2 CTAs per SM, INT8: 1)
    assert f(INT4, 1, 8, 32, 16, 8192, 0, 148) == 37
    assert f(INT8, 1, 8, 32, 16, 8192, 0, 148) == 18
    # FP8 and group 8 stay on the fp16-MMA kernel: 4 CTAs per SM, 32-token stages
    assert f(FP8, 1, 8, 32, 64, 2048, 0, 148) == 74
    assert f(INT4, 1, 8, 64, 64, 2048, 0, 148) == 74
    # INT4 with batch x kv_heads >= 256 and a block table of >= 32k tokens uses the 3-CTA/SM
    # tcgen05 shape (more splits than INT8); shorter tables and smaller batches keep 2 per SM
    assert f(INT4, 64, 8, 32, 64, 512, 0, 148) == 6
    assert f(INT4, 32, 8, 32, 64, 512, 0, 148) == 12
    assert f(INT4, 32, 8, 32, 64, 128, 0, 148) == 8
    assert f(INT8, 64, 8, 32, 64, 512, 0, 148) == 4
    assert f(INT4, 8, 8, 32, 64, 512, 0, 148) == 4
    # explicit requests are clamped to the 128-token chunk count
    assert f(INT4, 1, 8, 32, 64, 3, 50, 148) == 2
    assert f(INT4, 1, 8, 32, 64, 3, 1, 148) == 1


def test_workspace_bytes_monotone():
    from bpt.decode import workspace_bytes
    a = workspace_bytes(2, 32, 128, 1)
    b = workspace_bytes(2, 32, 128, 8)
    assert b > a >= 256
    assert b >= 256 + 2 * 32 * 8 * 128 * 4


def test_compute_entry_rejects_bad_arguments_without_gpu():
    lib = _lib.lib()
    rc = lib.bpt_decode_fp16(None, 0, 0, None, 0, 0, 0, None, 0, 0, 0, 0, None, 0, None, None,
                             0, 0, 1, 32, 7, 128, 16, 1, 0.0, 0, 148, None, 0, None)
    assert rc == _lib.ERR_INVALID_ARGUMENT  # Hq % Hkv != 0
    rc = lib.bpt_decode_fp16(None, 0, 0, None, 0, 0, 0, None, 0, 0, 0, 0, None, 0, None, None,
                             0, 0, 0, 32, 8, 128, 16, 1, 0.0, 0, 148, None, 0, None)
    assert rc == 0  # empty batch is a no-op
