"""TEST INFRASTRUCTURE ONLY — not part of the product.

CPU restatement (numpy) of the reference streaming atlas of haelyons/proteus. Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg may import this package, and only as the
checker or as the timed CPU baseline; the product path (proteus_b200) never imports it.

Pinning: the restatement is checked against golden vectors produced by the reference itself
(tests/golden/make_golden.py imports the reference's own `atlas` package and records its outputs;
tests/test_oracle_golden.py compares this oracle with them).
"""
