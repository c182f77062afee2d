"""CPU oracle for the UniCache physical-engine hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this
directory: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of
``bench.py`` (``cpu_baseline`` and ``--impl reference``) use it, and only as the
checker or the timed CPU baseline, never as the product path.

Each function restates, in numpy, the algorithm of the UniCache reference
implementation (Superone77/UniCache) and cites the file:line it follows:

* ``oracle.numerics``  bf16/fp16 rounding used by the reference's ``.to(dtype)``
* ``oracle.kivi``      KIVI grouped quantization, int32 bit-packing, dequant,
                       the packed-cache split, fake quantization
* ``oracle.attention`` GQA attention over dense/packed segments with LSE,
                       and the LSE merge of attention summaries
* ``oracle.h2o``       per-KV-head H2O selection, compaction, score
                       accumulation, trim and budget requests
* ``oracle.compact``   dense-cache keep-mask compaction

Parity pin: the oracle is checked bit-for-bit against golden vectors written
by ``tests/golden/make_golden.py``, which imports the reference's own Python
implementation (``unicache.storage.physical`` and friends) and records its
outputs (see ``tests/test_oracle_golden.py``).
"""
