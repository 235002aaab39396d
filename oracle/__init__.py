"""CPU oracle for the tensor-parallel paged Qwen2 layer.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
directory: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and only
as the checker or as the timed CPU baseline.

``qwen2_ref`` restates, in fp32 PyTorch on the CPU, the arithmetic of the
reference project's forward pass (``src/tinybatch/model.py``,
``src/tinybatch/kv_cache.py``, ``src/tinybatch/tensor_parallel.py``).  Each
function cites the reference lines it follows.  The restatement is pinned
against golden vectors produced by running the reference itself
(``tests/golden/make_golden.py``; checked by ``tests/test_oracle_golden.py``).
"""
