"""CPU oracle for the sf hot path.  TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the arithmetic of the reference
(aloshdenny/superfloat.python, package ``sf`` v0.16.0) for the data-parallel
hot path: the elementwise sfN ops with their event masks, the chain matmul
and the wide (MX engine) matmul with its POP rounding.  Every function cites
the reference file:line it restates.

It is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke``
and the CPU-baseline leg of ``bench.py`` may import it.  The product path
(``superfloat.python_b200``) never imports it and fails loudly when its CUDA
library is missing.

Pinning: ``tests/test_oracle.py`` checks these functions against the
reference's own golden vectors (spec/golden/*.json, spec/golden/wide/
dot_wide_shift.json, tests/data/mx_golden.json) re-emitted under
``tests/golden/`` by ``tests/golden/make_golden.py``, and against outputs of
the reference itself (checksums of seeded runs) recorded by the same script.
``oracle/_ref`` (built by ``oracle/build_ref.py`` when the reference tree is
present) is the reference's own C accumulator, used as a second check and as
the CPU baseline of the wide matmul.
"""
