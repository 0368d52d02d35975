"""CPU oracle for the paged-KV GQA decode path. TEST INFRASTRUCTURE ONLY.

Nothing in the shipped package (``kvq-decode_b200/bpt``) imports this directory. Only the
test suite, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` use it, and
only as the checker / the timed CPU reference, never as the thing measured or shipped.

Modules:
  attention  numpy fp32 restatement of ``paged_decode_attention_ref``
             (reference: src/bpt/reference.py:20-49)
  cache      seeded numpy paged-cache builder (reference: src/bpt/reference.py:52-82) plus
             the BASELINE workload generators (spare blocks, zero-padded block tables,
             uniform ragged lengths, outlier key channels)
  kivi       numpy KIVI quantizer / dequantizer: the bit-exact specification of the INT8,
             FP8-E4M3 and INT4 cache formats (no reference counterpart: parity unpinned by
             the reference, pinned by this spec and committed golden codes)

Pinning: ``tests/golden/make_golden.py`` runs the reference's own
``paged_decode_attention_ref`` (torch, CPU) on inputs generated here and commits the outputs;
``tests/test_oracle_golden.py`` checks this oracle against them.
"""
