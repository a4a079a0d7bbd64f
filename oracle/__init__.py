"""Test infrastructure: CPU restatement of the reference algorithm (parity oracle).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs
import this package; the product package never does.
"""
