"""Parity oracle — TEST INFRASTRUCTURE ONLY.

CPU restatements of the reference's router and ternary-expert math, used as
the checker by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg
of ``bench.py``.  Nothing in the product package imports this module; the
CUDA path never routes through it.

Pinning: ``tests/golden/*.npz`` were produced by running the reference's own
Python modules (``tests/golden/make_golden.py``); ``tests/test_oracle.py``
checks these restatements against them.
"""
