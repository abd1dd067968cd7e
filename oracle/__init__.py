"""CPU oracle of PagedCore's paged KV-cache hot path - TEST INFRASTRUCTURE ONLY.

A restatement of the reference algorithms (src/pagedcore/kv_cache.py,
attention.py and dense.py of Anassbzdd/PagedCore) in plain Python and numpy,
used as the checker of the B200 implementation.  Only tests/, the
``smoke()`` check of __graft_entry__ and the CPU-baseline leg of bench.py may
import it; the product package never does.

Parity pinning: the oracle is checked against golden vectors produced by
running the reference itself (tests/golden/make_golden.py imports the
reference's own modules), and against the known-answer cases of the
reference's unit tests.

Modules:
- ``allocator``  KVAllocator bookkeeping (LIFO free list, credits, staged decode).
- ``rope``       the FP16 cos/sin table and the FP16 rotation of apply_rope.
- ``kv_write``   append / write_decode_layer into a numpy FP16 pool.
- ``attention``  paged_attention's page loop in FP32, and an FP64 dense reference.
- ``torch_decoder``  the reference's contiguous FP32-attention decoder and its
  FP32 page loop in torch, to compare the decoder on the same GPU.
"""
