"""Drop-in names of the reference module ``bpt.triton_fp16`` (src/bpt/triton_fp16.py).

Code written against the reference keeps working unchanged:

    from bpt.triton_fp16 import paged_decode_attention_triton, choose_num_splits, _sm_count

Nothing here is Triton: every name resolves to the sm_100a CUDA implementation in
``bpt.decode``. The heuristic constants keep their reference names but describe the B200
planner (CTAs resident per SM, minimum tokens per split).
"""
from .decode import _sm_count, choose_num_splits, paged_decode_attention

# reference: src/bpt/triton_fp16.py:166-167 (values are the B200 planner's: one wave of
# 4 resident CTAs per SM when >= 4 splits of at most 8192 tokens fit, else just under 7
# waves; >= 2 chunks of 32 tokens)
TARGET_PROGRAMS_PER_SM = 4
MIN_TOKENS_PER_SPLIT = 64

paged_decode_attention_triton = paged_decode_attention

__all__ = ["paged_decode_attention_triton", "choose_num_splits", "_sm_count",
           "TARGET_PROGRAMS_PER_SM", "MIN_TOKENS_PER_SPLIT"]
