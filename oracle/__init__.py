"""CPU oracle for the ragged paged-attention path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU and in plain torch/Python, the algorithm of
nifre's paged KV cache and cached attention (jyotilakra92/nifre, files under
``src/inference/``).  It exists to check the CUDA path; it is never the thing
measured or shipped.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference`` arm) may import
it.  The product package ``nifre_b200`` never imports it and has no CPU
fallback.

Pinning: every function here is checked against golden fixtures in
``tests/golden/`` that were produced by running the reference implementation
itself (``tests/golden/make_golden.py`` imports the reference's own
``src/inference`` modules).  ``tests/test_oracle_golden.py`` holds those checks.
The reference pins attention numerics only through its own torch version; the
fixtures record the outputs of that code on this image's torch 2.11.

Modules
-------
paged      -- block allocator, block table, prefix index, paged KV store
              (reference ``block_allocator.py``, ``block_table.py``,
              ``prefix_cache.py``, ``paged_kv_cache.py``)
attention  -- cached causal attention per row, with grouped-query heads
              expanded by ``repeat_interleave`` (reference ``attention.py``)
engine     -- greedy generation one request at a time (reference
              ``engine.py``/``model_runner.py`` semantics), for the
              end-to-end configuration's tokens and CPU baseline
"""
