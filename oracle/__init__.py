"""Oracle: CPU (and torch-op) restatements of the reference's hot path.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference leg may import anything from this
package, and only as the checker or as the timed stand-in for the
reference's own CPU path. The product (``cascade-llm_b200/``) never imports
it; the product fails loudly when its CUDA library is missing.

Parity pins: ``tests/golden/`` holds vectors produced by running the
reference's own ``layer_streaming`` code (see ``tests/golden/make_golden.py``);
``tests/test_oracle_golden.py`` checks every restatement here against them.
"""
