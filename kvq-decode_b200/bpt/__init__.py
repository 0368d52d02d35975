"""bpt — B200-native paged-KV GQA decode attention (sm_100a CUDA behind a C ABI).

Public API (the reference project's ``bpt`` names are kept where they exist):

  paged_decode_attention(q, k_cache, v_cache, block_table, seq_lens, scale=None,
                         num_splits=None)              FP16 cache
  bpt.triton_fp16.paged_decode_attention_triton        the reference's name for the same call
  bpt.cache.build_paged_cache                          reference test-cache builder (torch)
  bpt.roofline                                         bytes-per-token / roofline model + CLI

There is no CPU or Triton fallback: compute entry points need CUDA tensors and the in-tree
library ``bpt/libbpt_b200.so`` (built by ``kvq-decode_b200/build.py``).
"""
from ._lib import BptArgumentError, BptError, BptUnsupportedError
from .cache import build_paged_cache
from .decode import choose_num_splits, paged_decode_attention

__all__ = ["paged_decode_attention", "choose_num_splits", "build_paged_cache", "BptError",
           "BptArgumentError", "BptUnsupportedError"]
__version__ = "0.1.0"
