"""CPU restatement of LinkQ2's W4A16 and KV4 arithmetic.

TEST INFRASTRUCTURE ONLY.  Nothing under this package is part of the product:
the shipped operators live in ``linkq2_b200`` and run on the GPU through the
C-ABI library.  This package is imported by the test-suite, by the smoke check
and by the CPU-baseline leg of the benchmark, and nowhere else.

Every function cites the reference file and lines it restates (paths are
relative to the LinkQ2 project root).  The restatement is pinned against
outputs of the reference itself: ``tests/golden/make_golden.py`` imports the
reference (its Triton kernels under the Triton CPU interpreter) and stores
small input/output fixtures that ``tests/test_oracle_golden.py`` replays
against this package.
"""
from . import kv4, w4a16  # noqa: F401
