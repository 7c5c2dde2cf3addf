"""Test infrastructure: the CPU parity oracle and synthetic-checkpoint generator.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
import this package. The product library never does.
"""
