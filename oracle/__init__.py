"""CPU oracle for the cache-aware FastConformer streaming hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
directory; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of
``bench.py`` (``cpu_baseline`` and ``--impl reference``) use it, and only as
the checker or as the timed CPU restatement of the reference.

It is a float64/int64 numpy restatement of the reference's algorithm for the
path (odunola499/parakeet-streaming):

* ``streaming``  - dense per-slot window cache, shift-append, conv cache,
  streaming masks, rel-pos table, ``rel_shift``, rel-pos MHSA, causal
  depthwise conv module, Conformer layer and encoder step, and the slot
  scheduler's FIFO free list (``parakeet/modules/cache.py``,
  ``parakeet/modules/encoder.py``, ``parakeet/modules/attention.py``,
  ``parakeet/modules/convolution.py``, ``parakeet/engine/scheduler.py``).
* ``pages``      - CPU model of the page allocator and paged window that
  the CUDA path implements.  The reference has no pages (its pool is one
  dense window per slot), so page-id values are pinned by this model, and
  window contents are pinned against the reference's dense windows.

Parity pin: every restated function is checked against golden vectors that
``tests/golden/make_golden.py`` produced by running the reference's own
modules on seeded inputs (``tests/test_oracle_golden.py``).
"""
