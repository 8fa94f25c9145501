"""CPU oracle for the W8A8 bposit path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference's arithmetic for the hot
path (int8 quantisation, exact INT32 GEMM, quire256 -> bposit16/32 encoders,
bposit16 decode/quire sums, the bposit16 ALU tables).  It is the checker the
parity tests compare the CUDA library against, and the timed CPU baseline of
``bench.py``.  Nothing in the shipped library imports it; only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may use it.

Parity pinning: every function here is checked (tests/test_oracle_*.py)
against the golden vectors under ``tests/golden/`` that were produced from the
reference's own Python implementation (kernels/bposit16_reference.py) and
its known-answer tables, and against the reference's published SHA-256 probe
hashes of the W8A8 fp32 output.
"""
