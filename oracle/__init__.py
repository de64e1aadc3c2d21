"""ORACLE — test infrastructure, never part of the product.

CPU restatements of the reference's paged INT8 KV-cache path, used only by
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg as
the checker.  Nothing under ``llm-inference-accelerator_b200/`` imports this
package.

Modules:
  quant         per-head symmetric INT8 quantizer (C restatement + numpy),
                follows native/src/native.cpp:275-353 and
                src/specdecode/kv_cache.py:119-151
  paged_cache   allocator / append / truncate state machine with device-layout
                storage, follows src/specdecode/kv_cache.py:201-473 and the
                slot clearing of src/specdecode/cuda_kv_cache.py:333-354
  attention     fp64 restatement and a CPU-torch restatement of the reference's
                unfused paged attention, src/specdecode/cuda_kv_cache.py:452-497
  workloads     seeded synthetic inputs shaped like the benchmark configurations

Parity is pinned: tests/golden/ holds vectors produced by running the
reference itself (its Python package and its C++ library compiled from its own
sources by oracle/Makefile), and tests/test_oracle_golden.py checks this
package against them.
"""
