"""ctypes binding of the bpt C ABI (include/bpt.h) and the status -> exception mapping.

The shared library is built in-tree by ``kvq-decode_b200/build.py`` as
``bpt/libbpt_b200.so``. There is no fallback: if the library is missing or fails to load,
every compute entry point raises, loudly. Host-only helpers (split planner, workspace sizing)
go through the same library so Python and C++ can never disagree.
"""
import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("BPT_LIBRARY", os.path.join(_HERE, "libbpt_b200.so"))

_lock = threading.Lock()
_lib = None

c_i32, c_i64, c_f32, c_size, c_vp = (ctypes.c_int, ctypes.c_int64, ctypes.c_float,
                                     ctypes.c_size_t, ctypes.c_void_p)


class BptError(RuntimeError):
    """A bpt C-ABI call failed (launch error, driver error, device check)."""

    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = status_string(status) if _lib is not None else str(status)
        super().__init__(f"{what}: {msg} (status {status})" if what else msg)


class BptArgumentError(ValueError, AssertionError):
    """Invalid arguments. Subclasses AssertionError because the reference's launcher
    validates with ``assert`` (src/bpt/triton_fp16.py:195-201); callers that catch either
    ValueError or AssertionError keep working."""


class BptUnsupportedError(BptArgumentError):
    """A shape outside the built kernel set (head_dim, group, block_size)."""


# (name, restype, argtypes)
_SIGNATURES = [
    ("bpt_status_string", ctypes.c_char_p, [c_i32]),
    ("bpt_version", c_i32, []),
    ("bpt_plan_splits", c_i32, [c_i32, c_i32, c_i32, c_i32, c_i32]),
    ("bpt_effective_splits", c_i32, [c_i32, c_i32, c_i32, c_i32, c_i32, c_i32]),
    ("bpt_decode_workspace_bytes", c_size, [c_i32, c_i32, c_i32, c_i32]),
    ("bpt_decode_fp16", c_i32,
     [c_vp, c_i64, c_i64,                      # q, q_sb, q_sh
      c_vp, c_i64, c_i64, c_i64,               # k_cache + strides
      c_vp, c_i64, c_i64, c_i64,               # v_cache + strides
      c_i64,                                   # num_blocks
      c_vp, c_i64,                             # block_table, bt_sb
      c_vp,                                    # seq_lens
      c_vp, c_i64, c_i64,                      # out, o_sb, o_sh
      c_i32, c_i32, c_i32, c_i32,              # batch, q_heads, kv_heads, head_dim
      c_i32, c_i32,                            # block_size, max_blocks
      c_f32, c_i32, c_i32,                     # scale, num_splits, sm_count
      c_vp, c_size, c_vp]),                    # workspace, bytes, stream
    ("bpt_decode_fp16_partial", c_i32,
     [c_vp, c_i64, c_i64,
      c_vp, c_i64, c_i64, c_i64,
      c_vp, c_i64, c_i64, c_i64,
      c_i64, c_vp, c_i64, c_vp,
      c_i32, c_i32, c_i32, c_i32, c_i32, c_i32,  # batch, Hq, Hkv, D, block_size, max_blocks
      c_f32, c_i32,                              # scale, splits
      c_vp, c_vp, c_vp, c_vp]),                  # o_part, lse, status, stream
    ("bpt_merge_partials", c_i32,
     [c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_i64, c_i64, c_vp]),
    ("bpt_merge_states", c_i32,
     [c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp]),
    ("bpt_selftest_wait_timeout", c_i32, [c_vp, ctypes.c_uint, c_vp]),
]

# Status codes (include/bpt.h enum bpt_status)
OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED_SHAPE = -2
ERR_WORKSPACE_TOO_SMALL = -3
ERR_ALIGNMENT = -6


def lib() -> ctypes.CDLL:
    """Load (once) and return the library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"bpt CUDA library not found at {LIB_PATH}; build it with "
                    "`python kvq-decode_b200/build.py` (there is no CPU fallback)")
            handle = ctypes.CDLL(LIB_PATH)
            for name, res, args in _SIGNATURES:
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def register(name, restype, argtypes):
    """Declare an additional entry point's signature (used by the other modules)."""
    fn = getattr(lib(), name)
    fn.restype = restype
    fn.argtypes = argtypes
    return fn


def status_string(status: int) -> str:
    return lib().bpt_status_string(int(status)).decode()


def check(status: int, what: str):
    if status == OK:
        return
    if status == ERR_UNSUPPORTED_SHAPE:
        raise BptUnsupportedError(f"{what}: {status_string(status)}")
    if status in (ERR_INVALID_ARGUMENT, ERR_WORKSPACE_TOO_SMALL, ERR_ALIGNMENT):
        raise BptArgumentError(f"{what}: {status_string(status)}")
    raise BptError(status, what)
