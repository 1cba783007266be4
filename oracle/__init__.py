"""CPU oracle for the BF16 projection path. TEST INFRASTRUCTURE ONLY.

Nothing in the product (the ``muse_bf16_proj_b200`` package, its CUDA library, ``bench.py``'s GPU
arms) imports, links or runs this package. Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline / reference legs of ``bench.py`` use it, and only as the checker or as the timed CPU
restatement of the reference's own CPU path.

Modules:

- ``contract_ref``: the reference's FP64 product and output checks (reference.py:72-99,
  checks.py:14-55) restated in numpy.
- ``codec12_ref``: the reference's 12-bit weight packing (submission.py:591-626, per-layer window
  base) and the build's per-tile-base 12-bit format, restated in numpy.

Pinning: both are checked in ``tests/test_oracle_golden.py`` against fixtures that
``tests/golden/make_golden.py`` produced by importing the reference's own ``reference.py`` and
``submission.py`` on the CPU (hashes of the reference's generated weights, inputs, FP64 outputs and
12-bit planes, plus literal small cases).
"""
